// Row-wise kernels of the token-batch path: LayerNorm + token shift + lerp mixes,
// the final LayerNorm of logit rows, and the state-x write-back.
//
// One CTA per token row, C/4 threads, 4 channels (8 bytes) per thread.
// Token shift: the previous token of row m is row m-1 when both belong to the
// same sequence, else the sequence's saved state x (demo/_rwkv7_base.py:228-229).
#include "common.cuh"

namespace {

// Block-wide sums of NV values per thread with the rounding of the layout of one
// thread per 4 channels: a thread holds P partials (each the in-order sum over its 4
// channels: the "4-channel threads" P * t .. P * t + P - 1). The 32-lane butterfly of
// each 4-channel warp is replayed (offsets >= P as shuffles, smaller ones within the
// thread), then the 4-channel warps' totals are added in order. blockDim.x * P must be
// a multiple of 32.
template <int P, int NV>
__device__ __forceinline__ void block_sum_p(float (&v)[NV][P], float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (int)(blockDim.x * P + 31) >> 5;  // 4-channel warps
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (off >= P) {
#pragma unroll
        for (int q = 0; q < P; ++q) v[i][q] += __shfl_xor_sync(0xffffffffu, v[i][q], off / P);
      } else {
        float t[P];
#pragma unroll
        for (int q = 0; q < P; ++q) t[q] = v[i][q] + v[i][q ^ off];
#pragma unroll
        for (int q = 0; q < P; ++q) v[i][q] = t[q];
      }
    }
  }
  __syncthreads();
  if (((P * lane) & 31) == 0) {
    const int w4 = (P * (32 * wid + lane)) >> 5;
#pragma unroll
    for (int i = 0; i < NV; ++i) red[w4 * NV + i] = v[i][0];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float s = 0.f;
    for (int w = 0; w < nw; ++w) s += red[w * NV + i];
#pragma unroll
    for (int q = 0; q < P; ++q) v[i][q] = s;
  }
  __syncthreads();
}

// LayerNorm of NROW rows already in registers (P groups of 4 channels per thread,
// group q at channel c + 4q), fp32 math, output rounded to fp16 like F.layer_norm on
// an fp16 tensor (weight.py:6-15).
template <int NROW, int P>
__device__ __forceinline__ void ln_rows(float4 (&x)[NROW][P], const __half* w, const __half* b,
                                        int c, int C, float* red) {
  float s[NROW][P];
#pragma unroll
  for (int i = 0; i < NROW; ++i)
#pragma unroll
    for (int q = 0; q < P; ++q) s[i][q] = x[i][q].x + x[i][q].y + x[i][q].z + x[i][q].w;
  block_sum_p<P, NROW>(s, red);
  float mean[NROW];
#pragma unroll
  for (int i = 0; i < NROW; ++i) {
    mean[i] = s[i][0] / C;
#pragma unroll
    for (int q = 0; q < P; ++q) {
      const float dx = x[i][q].x - mean[i], dy = x[i][q].y - mean[i], dz = x[i][q].z - mean[i],
                  dw = x[i][q].w - mean[i];
      s[i][q] = dx * dx + dy * dy + dz * dz + dw * dw;
    }
  }
  block_sum_p<P, NROW>(s, red);
#pragma unroll
  for (int q = 0; q < P; ++q) {
    const float4 ww = load_h4(w + c + 4 * q), bb = load_h4(b + c + 4 * q);
#pragma unroll
    for (int i = 0; i < NROW; ++i) {
      const float rstd = rsqrtf(s[i][0] / C + 1e-5f);
      x[i][q].x = r16((x[i][q].x - mean[i]) * rstd * ww.x + bb.x);
      x[i][q].y = r16((x[i][q].y - mean[i]) * rstd * ww.y + bb.y);
      x[i][q].z = r16((x[i][q].z - mean[i]) * rstd * ww.z + bb.z);
      x[i][q].w = r16((x[i][q].w - mean[i]) * rstd * ww.w + bb.w);
    }
  }
}

// out = x + mu * (prev - x) with the reference's fp16 rounding points.
template <int SEM>
__device__ __forceinline__ float lerp_sem(float x, float prev, float mu) {
  const float diff = r16(prev - x);
  if (SEM == SEM_DECODE) return r16(x + mu * diff);  // lerp.py:106-114 (fused fp16 fma)
  return r16(x + r16(mu * diff));                   // _rwkv7_base.py:230-236 (two torch ops)
}

template <int SEM>
__device__ __forceinline__ float4 lerp4(float4 x, float4 p, float4 mu) {
  return make_float4(lerp_sem<SEM>(x.x, p.x, mu.x), lerp_sem<SEM>(x.y, p.y, mu.y),
                     lerp_sem<SEM>(x.z, p.z, mu.z), lerp_sem<SEM>(x.w, p.w, mu.w));
}

// Row m, channels c..c+3, of a residual sum whose split-K reduce was left to this
// kernel: fp16(res + fp16(sum_s ws[s])), slices summed in split order -- the same
// values the GEMM's residual epilogue (RWKV_EPI_RESID) stores after its reduce.
__device__ __forceinline__ float4 pending_row4(const PendingResid& p, int m, int c, int M, int C) {
  const size_t i = (size_t)m * C + c, MC = (size_t)M * C;
  float4 acc = __ldcg(reinterpret_cast<const float4*>(p.ws + i));
  for (int s = 1; s < p.splits; ++s) {
    const float4 q = __ldcg(reinterpret_cast<const float4*>(p.ws + s * MC + i));
    acc.x += q.x; acc.y += q.y; acc.z += q.z; acc.w += q.w;
  }
  const float4 r = load_h4(p.res + i);
  return make_float4(r16(r.x + r16(acc.x)), r16(r.y + r16(acc.y)), r16(r.z + r16(acc.z)),
                     r16(r.w + r16(acc.w)));
}

}  // namespace

// P groups of 4 channels at p + 4q: one 16-byte access per thread for P = 2 (workspace
// rows only: 16-byte aligned), 8-byte accesses otherwise.
template <int P>
__device__ __forceinline__ void load_rows(const __half* p, float4 (&v)[P]) {
  if constexpr (P == 2) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    const float2 a = __half22float2(h[0]), b = __half22float2(h[1]), c = __half22float2(h[2]),
                 d = __half22float2(h[3]);
    v[0] = make_float4(a.x, a.y, b.x, b.y);
    v[1] = make_float4(c.x, c.y, d.x, d.y);
  } else {
#pragma unroll
    for (int q = 0; q < P; ++q) v[q] = load_h4(p + 4 * q);
  }
}
template <int P>
__device__ __forceinline__ void store_rows(__half* p, const float4 (&v)[P]) {
  if constexpr (P == 2) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
    h[0] = __floats2half2_rn(v[0].x, v[0].y);
    h[1] = __floats2half2_rn(v[0].z, v[0].w);
    h[2] = __floats2half2_rn(v[1].x, v[1].y);
    h[3] = __floats2half2_rn(v[1].z, v[1].w);
    *reinterpret_cast<uint4*>(p) = u;
  } else {
#pragma unroll
    for (int q = 0; q < P; ++q) store_h4(p + 4 * q, v[q]);
  }
}
// Caller memory (embedding rows, state x, mix vectors): 8-byte accesses.
template <int P>
__device__ __forceinline__ void load_user(const __half* p, float4 (&v)[P]) {
#pragma unroll
  for (int q = 0; q < P; ++q) v[q] = load_h4(p + 4 * q);
}

// Row kernels: one CTA per token row, C / (4P) threads, 4P channels per thread (P = 1
// for small batches, P = 2 -- 16-byte accesses, twice the rows in flight per SM -- for
// large ones); LayerNorm sums round the same for both.

// TMIX input stage: [embedding gather] + LN1 + token shift + 6 lerps.
//   x      : [M, C] layer input (written here when `tokens` != NULL: layer 0 gathers emb rows)
//   xmix   : 6 x [M, C] = xr, xw, xk, xv, xa, xg
//   xlast  : [S, C] LN1 output of each sequence's last row (new state x)
template <int SEM, int P>
__global__ void k_tmix_rows(__half* __restrict__ x, const int64_t* __restrict__ tokens,
                            const __half* __restrict__ emb, const __half* __restrict__ ln_w,
                            const __half* __restrict__ ln_b, const __half* __restrict__ mix6,
                            const __half* __restrict__ state_x, const int* __restrict__ row_seq,
                            const int* __restrict__ cu, const int* __restrict__ slots,
                            __half* __restrict__ xmix, __half* __restrict__ xlast, int M, int C,
                            const PendingResid pend) {
  RWKV_GRID_DEP_ENTRY();
  __shared__ float red[32 * 2];
  const int m = blockIdx.x, c = threadIdx.x * 4 * P;
  const int s = row_seq[m];
  const bool first = (m == cu[s]), last = (m == cu[s + 1] - 1);
  float4 v[2][P];
  if (tokens) {
    load_user<P>(emb + (size_t)tokens[m] * C + c, v[0]);
    if (!first) load_user<P>(emb + (size_t)tokens[m - 1] * C + c, v[1]);
    store_rows<P>(x + (size_t)m * C + c, v[0]);
  } else if (pend.ws) {  // x = res + (split-K GEMM output), finished here
#pragma unroll
    for (int q = 0; q < P; ++q) {
      v[0][q] = pending_row4(pend, m, c + 4 * q, M, C);
      if (!first) v[1][q] = pending_row4(pend, m - 1, c + 4 * q, M, C);
    }
    store_rows<P>(x + (size_t)m * C + c, v[0]);
  } else {
    load_rows<P>(x + (size_t)m * C + c, v[0]);
    if (!first) load_rows<P>(x + (size_t)(m - 1) * C + c, v[1]);
  }
  if (first) {
#pragma unroll
    for (int q = 0; q < P; ++q) v[1][q] = v[0][q];
  }
  ln_rows<2, P>(v, ln_w, ln_b, c, C, red);
  const int slot = slots ? slots[s] : s;
  float4 prev[P];
  if (first)
    load_user<P>(state_x + (size_t)slot * C + c, prev);
  else
#pragma unroll
    for (int q = 0; q < P; ++q) prev[q] = v[1][q];
  const size_t plane = (size_t)M * C;
#pragma unroll
  for (int j = 0; j < 6; ++j) {
    float4 mu[P], o[P];
    load_user<P>(mix6 + j * C + c, mu);
#pragma unroll
    for (int q = 0; q < P; ++q) o[q] = lerp4<SEM>(v[0][q], prev[q], mu[q]);
    store_rows<P>(xmix + j * plane + (size_t)m * C + c, o);
  }
  if (last) store_rows<P>(xlast + (size_t)s * C + c, v[0]);
}

// CMIX input stage: LN2 + token shift + one lerp (x_k).
template <int SEM, int P>
__global__ void k_cmix_rows(__half* __restrict__ x, const __half* __restrict__ ln_w,
                            const __half* __restrict__ ln_b, const __half* __restrict__ mu,
                            const __half* __restrict__ state_x, const int* __restrict__ row_seq,
                            const int* __restrict__ cu, const int* __restrict__ slots,
                            __half* __restrict__ xk, __half* __restrict__ xlast, int M, int C,
                            const PendingResid pend) {
  RWKV_GRID_DEP_ENTRY();
  __shared__ float red[32 * 2];
  const int m = blockIdx.x, c = threadIdx.x * 4 * P;
  const int s = row_seq[m];
  const bool first = (m == cu[s]), last = (m == cu[s + 1] - 1);
  float4 v[2][P];
  if (pend.ws) {  // x = res + (split-K GEMM output), finished here
#pragma unroll
    for (int q = 0; q < P; ++q) {
      v[0][q] = pending_row4(pend, m, c + 4 * q, M, C);
      if (!first) v[1][q] = pending_row4(pend, m - 1, c + 4 * q, M, C);
    }
    store_rows<P>(x + (size_t)m * C + c, v[0]);
  } else {
    load_rows<P>(x + (size_t)m * C + c, v[0]);
    if (!first) load_rows<P>(x + (size_t)(m - 1) * C + c, v[1]);
  }
  if (first) {
#pragma unroll
    for (int q = 0; q < P; ++q) v[1][q] = v[0][q];
  }
  ln_rows<2, P>(v, ln_w, ln_b, c, C, red);
  const int slot = slots ? slots[s] : s;
  float4 prev[P], mv[P], o[P];
  if (first)
    load_user<P>(state_x + (size_t)slot * C + c, prev);
  else
#pragma unroll
    for (int q = 0; q < P; ++q) prev[q] = v[1][q];
  load_user<P>(mu + c, mv);
#pragma unroll
  for (int q = 0; q < P; ++q) o[q] = lerp4<SEM>(v[0][q], prev[q], mv[q]);
  store_rows<P>(xk + (size_t)m * C + c, o);
  if (last) store_rows<P>(xlast + (size_t)s * C + c, v[0]);
}

// ln_out of the rows that produce logits: out[i] = LN(x[rows[i]]).
__global__ void k_ln_rows(const __half* __restrict__ x, const int* __restrict__ rows,
                          const __half* __restrict__ w, const __half* __restrict__ b,
                          __half* __restrict__ out, int M, int C, const PendingResid pend) {
  RWKV_GRID_DEP_ENTRY();
  __shared__ float red[32];
  const int i = blockIdx.x, c = threadIdx.x * 4;
  float4 v[1][1];
  v[0][0] = pend.ws ? pending_row4(pend, rows[i], c, M, C) : load_h4(x + (size_t)rows[i] * C + c);
  ln_rows<1, 1>(v, w, b, c, C, red);
  store_h4(out + (size_t)i * C + c, v[0][0]);
}

// Greedy ids from the head GEMM's per-row keys (EPI_ARGMAX).
__global__ void k_argmax_finish(const unsigned long long* __restrict__ keys, int64_t* __restrict__ ids,
                                int n) {
  RWKV_GRID_DEP_ENTRY();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  ids[i] = (int64_t)(0xFFFFFFFFu - (uint32_t)(keys[i] & 0xFFFFFFFFull));
}

// New state x of every layer: tmix_x[l][slot] = xlast[l][0][s], cmix_x[l][slot] = xlast[l][1][s].
// grid = (S, L, 2), block = C/4.
__global__ void k_scatter_state_x(const __half* __restrict__ xlast, __half* __restrict__ tmix_x,
                                  __half* __restrict__ cmix_x, const int* __restrict__ slots,
                                  int S, int n_slots, int C) {
  RWKV_GRID_DEP_ENTRY();
  const int s = blockIdx.x, l = blockIdx.y, which = blockIdx.z, c = threadIdx.x * 4;
  const int slot = slots ? slots[s] : s;
  const __half* src = xlast + (((size_t)l * 2 + which) * S + s) * C + c;
  __half* dst = (which ? cmix_x : tmix_x) + ((size_t)l * n_slots + slot) * C + c;
  *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(src);
}

// 8 channels per thread once the batch is large (and C / 8 is whole warps).
static bool rows_wide(int M, int C) { return rwkv_rows_wide(M, C); }

int launch_tmix_rows(int sem, __half* x, const int64_t* tokens, const __half* emb,
                     const __half* ln_w, const __half* ln_b, const __half* mix6,
                     const __half* state_x, const int* row_seq, const int* cu, const int* slots,
                     __half* xmix, __half* xlast, int M, int C, PendingResid pend,
                     cudaStream_t st) {
#define TMIX_GO(S, P)                                                                          \
  return rwkv_launch("tmix_rows", k_tmix_rows<S, P>, dim3(M), dim3(C / (4 * P)), 0, st, x,     \
                     tokens, emb, ln_w, ln_b, mix6, state_x, row_seq, cu, slots, xmix, xlast, M, \
                     C, pend)
  if (rows_wide(M, C)) {
    if (sem == SEM_DECODE) TMIX_GO(SEM_DECODE, 2);
    TMIX_GO(SEM_PREFILL, 2);
  }
  if (sem == SEM_DECODE) TMIX_GO(SEM_DECODE, 1);
  TMIX_GO(SEM_PREFILL, 1);
#undef TMIX_GO
}

int launch_cmix_rows(int sem, __half* x, const __half* ln_w, const __half* ln_b,
                     const __half* mu, const __half* state_x, const int* row_seq, const int* cu,
                     const int* slots, __half* xk, __half* xlast, int M, int C, PendingResid pend,
                     cudaStream_t st) {
#define CMIX_GO(S, P)                                                                          \
  return rwkv_launch("cmix_rows", k_cmix_rows<S, P>, dim3(M), dim3(C / (4 * P)), 0, st, x,     \
                     ln_w, ln_b, mu, state_x, row_seq, cu, slots, xk, xlast, M, C, pend)
  if (rows_wide(M, C)) {
    if (sem == SEM_DECODE) CMIX_GO(SEM_DECODE, 2);
    CMIX_GO(SEM_PREFILL, 2);
  }
  if (sem == SEM_DECODE) CMIX_GO(SEM_DECODE, 1);
  CMIX_GO(SEM_PREFILL, 1);
#undef CMIX_GO
}

int launch_ln_rows(const __half* x, const int* rows, const __half* w, const __half* b,
                   __half* out, int n, int M, int C, PendingResid pend, cudaStream_t st) {
  if (n == 0) return RWKV_OK;
  return rwkv_launch("ln_rows", k_ln_rows, dim3(n), dim3(C / 4), 0, st, x, rows, w, b, out, M, C,
                     pend);
}

int launch_argmax_finish(const unsigned long long* keys, int64_t* ids, int n, cudaStream_t st) {
  return rwkv_launch("argmax_finish", k_argmax_finish, dim3((n + 255) / 256), dim3(256), 0, st, keys,
                     ids, n);
}

int launch_scatter_state_x(const __half* xlast, __half* tmix_x, __half* cmix_x, const int* slots,
                           int S, int L, int n_slots, int C, cudaStream_t st) {
  return rwkv_launch("scatter_state_x", k_scatter_state_x, dim3(S, L, 2), dim3(C / 4), 0, st, xlast,
                     tmix_x, cmix_x, slots, S, n_slots, C);
}
