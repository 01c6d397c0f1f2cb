// Fused token sampling over [B, V] fp16 logits: one CTA of 1024 threads per row.
//
// Reference: sample_logits (demo/sampling.py:13-70): repetition penalty on the ids
// already generated (logit / p when > 0, * p otherwise), then greedy argmax when
// temperature <= 0; otherwise divide by the temperature, keep the top-k logits
// (every logit >= the k-th largest), keep the nucleus (a token survives when the
// softmax mass of the tokens ranked above it is <= top_p), and draw from the softmax
// of what is left. Differences, B200-side: one kernel per step instead of ~10 torch
// ops (topk, sort, cumsum, scatter, softmax, multinomial); the k-th largest value
// and the nucleus threshold come from radix selection on the logits' order-preserving
// integer keys (four 8-bit passes, histograms in shared memory) instead of sorting;
// the draw inverts the kept tokens' CDF, in a fixed order of the ids, at u * total for
// a caller-given uniform u in [0, 1) -- the same distribution as torch.multinomial,
// not the same stream of ids. Ties: every token tied with the k-th logit, and every token tied at
// the nucleus threshold, is kept (torch breaks such ties by its sort order).
// Masses are summed as 64-bit fixed-point integers, so every decision is
// bit-reproducible. V <= 65536 (the RWKV vocabulary).
#include "common.cuh"

namespace {

constexpr int ST = 1024;        // threads per row
constexpr int SPER = 64;        // ids per thread: thread t owns ids [64 t, 64 t + 64)
constexpr int SMAXV = ST * SPER;
constexpr double MASS_SCALE = 1099511627776.0;  // 2^40: fixed-point probability mass

// Order-preserving key of a float (larger float -> larger unsigned key).
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ unsigned long long mass_fx(float p) {
  return static_cast<unsigned long long>(__double2ll_rn((double)p * MASS_SCALE));
}

// Block-wide sum of one float per thread in a fixed order (bit-reproducible).
__device__ float block_sum_fixed(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x < 32) s = warp_sum(red[threadIdx.x]);
  if (threadIdx.x == 0) red[32] = s;
  __syncthreads();
  s = red[32];
  __syncthreads();
  return s;
}

__device__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float m = red[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) red[32] = m;
  }
  __syncthreads();
  const float m = red[32];
  __syncthreads();
  return m;
}

// Radix selection over the keys of the live ids (x > -inf). mode 0: the key of the
// k-th largest (count rank). mode 1: the nucleus threshold key -- the largest key t
// such that the mass of keys > t is <= top_p < mass of keys >= t (probabilities
// exp(x - m) * inv_s, in fixed point). Returns 0 when nothing is to be cut.
template <int MODE, typename Val>
__device__ uint32_t radix_select(Val&& val, unsigned long long dead, float m, float inv_s,
                                 long long k_or_unused, unsigned long long budget,
                                 unsigned long long* hist) {
  uint32_t prefix = 0, pmask = 0;
  unsigned long long above = 0;  // count (mode 0) or mass (mode 1) of keys above the prefix
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += ST) hist[i] = 0;
    __syncthreads();
    for (int i = 0; i < SPER; ++i) {
      if ((dead >> i) & 1ull) continue;
      const float xi = val(i);
      const uint32_t key = fkey(xi);
      if ((key & pmask) != prefix) continue;
      atomicAdd(&hist[(key >> shift) & 255u], MODE == 0 ? 1ull : mass_fx(expf(xi - m) * inv_s));
    }
    __syncthreads();
    // walk the bins from the top (one thread; 256 bins)
    __shared__ uint32_t s_bin;
    __shared__ unsigned long long s_above;
    if (threadIdx.x == 0) {
      unsigned long long acc = above;
      int b = 255;
      for (; b > 0; --b) {
        const unsigned long long nxt = acc + hist[b];
        if (MODE == 0 ? nxt >= (unsigned long long)k_or_unused : nxt > budget) break;
        acc = nxt;
      }
      s_bin = (uint32_t)b;
      s_above = acc;
    }
    __syncthreads();
    prefix |= s_bin << shift;
    pmask |= 255u << shift;
    above = s_above;
    __syncthreads();
  }
  return prefix;
}

__global__ void __launch_bounds__(ST, 1) k_sample(const __half* __restrict__ logits, int V,
                                                  float temperature, int top_k, float top_p,
                                                  float rep_penalty,
                                                  const int64_t* __restrict__ seen,
                                                  const int* __restrict__ seen_cu,
                                                  const float* __restrict__ uniforms,
                                                  int64_t* __restrict__ out) {
  extern __shared__ __align__(16) __half srow[];  // the row's logits [V]
  __shared__ uint32_t seen_bits[SMAXV / 32];
  __shared__ float red[33];
  __shared__ unsigned long long hist[256];
  __shared__ float tsum[ST];
  __shared__ unsigned long long s_pick;  // picked id + 1 (0: none yet)
  const int row = blockIdx.x, tid = threadIdx.x;
  const __half* lg = logits + (size_t)row * V;
  // thread t owns ids t + 1024 i (i < 64): coalesced, bank-conflict free
  for (int j = tid; j < V / 8; j += ST)
    reinterpret_cast<uint4*>(srow)[j] = reinterpret_cast<const uint4*>(lg)[j];
  // repetition penalty: ids of this row's seen list, as a bitmap (duplicates apply once)
  const bool pen = rep_penalty != 1.0f && seen && seen_cu;
  if (pen) {
    for (int i = tid; i < SMAXV / 32; i += ST) seen_bits[i] = 0;
    __syncthreads();
    for (int i = seen_cu[row] + tid; i < seen_cu[row + 1]; i += ST) {
      const int64_t id = seen[i];
      if (id >= 0 && id < V) atomicOr(&seen_bits[id >> 5], 1u << (id & 31));
    }
  }
  __syncthreads();
  unsigned long long dead = 0, pbit = 0;  // per owned id: masked out / penalised
#pragma unroll
  for (int i = 0; i < SPER; ++i) {
    const int id = tid + ST * i;
    if (id >= V) dead |= 1ull << i;
    else if (pen && ((seen_bits[id >> 5] >> (id & 31)) & 1u)) pbit |= 1ull << i;
  }
  auto val = [&](int i) -> float {
    float l = __half2float(srow[tid + ST * i]);
    if ((pbit >> i) & 1ull) l = l > 0.f ? l / rep_penalty : l * rep_penalty;
    return temperature > 0.f ? l / temperature : l;  // reference: l / temperature
  };
  if (!(temperature > 0.f)) {  // greedy: argmax, lowest id among equal values
    unsigned long long best = 0;
    for (int i = 0; i < SPER; ++i) {
      if ((dead >> i) & 1ull) continue;
      const unsigned long long key = ((unsigned long long)fkey(val(i)) << 32) |
                                     (unsigned long long)(0xFFFFFFFFu - (uint32_t)(tid + ST * i));
      best = key > best ? key : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
      best = t > best ? t : best;
    }
    if ((tid & 31) == 0) hist[tid >> 5] = best;
    __syncthreads();
    if (tid == 0) {
      unsigned long long b = 0;
      for (int w = 0; w < ST / 32; ++w) b = hist[w] > b ? hist[w] : b;
      out[row] = (int64_t)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
    }
    return;
  }
  if (top_k > 0 && top_k < V) {
    const uint32_t kth = radix_select<0>(val, dead, 0.f, 0.f, top_k, 0, hist);
    for (int i = 0; i < SPER; ++i)
      if (!((dead >> i) & 1ull) && fkey(val(i)) < kth) dead |= 1ull << i;
  }
  // softmax of the live logits
  float m = -INFINITY;
  for (int i = 0; i < SPER; ++i)
    if (!((dead >> i) & 1ull)) m = fmaxf(m, val(i));
  m = block_max(m, red);
  float s = 0.f;
  for (int i = 0; i < SPER; ++i)
    if (!((dead >> i) & 1ull)) s += expf(val(i) - m);
  s = block_sum_fixed(s, red);
  if (top_p < 1.0f) {
    const unsigned long long budget = mass_fx(top_p);
    const uint32_t thr = radix_select<1>(val, dead, m, 1.0f / s, 0, budget, hist);
    float s2 = 0.f;
    for (int i = 0; i < SPER; ++i) {
      if ((dead >> i) & 1ull) continue;
      const float xi = val(i);
      if (fkey(xi) < thr) dead |= 1ull << i;
      else s2 += expf(xi - m);
    }
    s = block_sum_fixed(s2, red);
  }
  // Inverse CDF over the live ids in a fixed order (thread-major: thread t's ids
  // t, t + 1024, ... then thread t + 1's): any fixed order draws the same
  // distribution. Thread sums, an exclusive scan in fixed order, then the owner walks.
  float mine = 0.f;
  int last_live = -1;
  for (int i = 0; i < SPER; ++i)
    if (!((dead >> i) & 1ull)) {
      mine += expf(val(i) - m);
      last_live = tid + ST * i;
    }
  tsum[tid] = mine;
  if (tid == 0) s_pick = 0;
  __syncthreads();
  if (tid < 32) {  // 32 thread sums per lane in order, then a lane prefix
    float run = 0.f;
    for (int j = 0; j < 32; ++j) run += tsum[tid * 32 + j];
    float incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, incl, o);
      if (tid >= o) incl += t;
    }
    float pre = incl - run;
    for (int j = 0; j < 32; ++j) {
      const float t = tsum[tid * 32 + j];
      tsum[tid * 32 + j] = pre;  // exclusive prefix
      pre += t;
    }
  }
  __syncthreads();
  float u = uniforms[row];
  u = fminf(fmaxf(u, 0.f), 0.99999994f);
  const float target = u * s;
  const float lo = tsum[tid];
  const float hi = tid + 1 < ST ? tsum[tid + 1] : s;
  if (mine > 0.f && target >= lo && target < hi) {
    float run = lo;
    int pick = last_live;  // float rounding can leave run <= target: take the last live id
    for (int i = 0; i < SPER; ++i) {
      if ((dead >> i) & 1ull) continue;
      run += expf(val(i) - m);
      if (run > target) { pick = tid + ST * i; break; }
    }
    atomicMax(&s_pick, (unsigned long long)pick + 1);
  }
  // fallback when rounding put the target past every range: the last live id in the
  // order, i.e. the last live id of the highest thread that has one
  int key = last_live < 0 ? -1 : tid * SPER + last_live / ST;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
  if ((tid & 31) == 0) reinterpret_cast<int*>(red)[tid >> 5] = key;
  __syncthreads();
  if (tid == 0) {
    long long p = (long long)s_pick - 1;
    if (p < 0) {
      int k = -1;
      for (int w = 0; w < ST / 32; ++w) k = max(k, reinterpret_cast<int*>(red)[w]);
      p = k < 0 ? 0 : (k / SPER) + ST * (k % SPER);
    }
    out[row] = p;
  }
}

}  // namespace

extern "C" int rwkv7_sample(const void* logits, int B, int V, float temperature, int top_k,
                            float top_p, float repetition_penalty, const int64_t* seen,
                            const int* seen_cu, const float* uniforms, int64_t* out,
                            void* stream) {
  rwkv_chain_begin();
  if (!logits || !out || B <= 0 || V <= 0 || V > SMAXV || (V & 7) ||
      (reinterpret_cast<uintptr_t>(logits) & 15)) {
    rwkv_set_error("rwkv7_sample: null pointer or bad size (B=%d, V=%d; V <= %d, a multiple of "
                   "8, logits 16-byte aligned)", B, V, SMAXV);
    return RWKV_ERR_ARG;
  }
  if (temperature > 0.f && !uniforms) {
    rwkv_set_error("rwkv7_sample: temperature > 0 needs one uniform per row");
    return RWKV_ERR_ARG;
  }
  if (top_k < 0 || !(top_p >= 0.f) || !(repetition_penalty > 0.f)) {
    rwkv_set_error("rwkv7_sample: top_k >= 0, top_p >= 0 and repetition_penalty > 0 required");
    return RWKV_ERR_ARG;
  }
  const size_t smem = (size_t)V * 2;
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      rwkv_set_error("rwkv7_sample: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return RWKV_ERR_CUDA;
    }
  }
  return rwkv_launch("sample", k_sample, dim3(B), dim3(ST), smem, (cudaStream_t)stream,
                     (const __half*)logits, V, temperature, top_k, top_p, repetition_penalty,
                     seen, seen_cu, uniforms, out);
}
