// Chunk-parallel wkv7 for prefill (many tokens per sequence).
//
// The serial recurrence S_t = S_{t-1} (diag(w_t) + a_t b_t^T) + v_t k_t^T,
// y_t = S_t r_t (src/rwkv_tl/kernels/dplr.py:174-227) is regrouped into chunks
// of L = 16 tokens. With G_t = sum_{i<=t} log w_i (per key column) and the
// decay-scaled vectors
//   at_t = a_t e^{G_{t-1}},  bh_j = b_j e^{-G_j},  kh_j = k_j e^{-G_j},  rt_t = r_t e^{G_t},
// every row s of the state (one value index) obeys, inside a chunk,
//   sa_t = s0 . at_t + sum_{j<t} (at_t . bh_j) sa_j + sum_{j<t} (at_t . kh_j) v_j
//   y_t  = s0 . rt_t + sum_{j<=t} (rt_t . bh_j) sa_j + (rt_t . kh_j) v_j
//   s_L  = s0 e^{G_L} + sum_j sa_j bh_j e^{G_L} + v_j kh_j e^{G_L}
// i.e. with T = (I - A_ab)^{-1} (A_ab strictly lower, unit-diagonal inverse):
//   sa = What s0 + PU v,   y = Q s0 + PY v,   s_L = s0 * gL + sa^T Bt + v^T Kt
//   What = T At, PU = T A_ak, Q = Rt + B_rb What, PY = B_rb PU + B_rk,
//   Bt = Bh e^{G_L}, Kt = Kh e^{G_L}, gL = e^{G_L}.
// All of it is state-independent, so k_chunk_prep runs in parallel over every
// (chunk, head); k_chunk_scan then walks the chunks of each sequence in order
// with the fp32 state of 8 rows in registers (one warp per row). All math is
// fp32; exponents stay within one chunk (|G| <= 16 * 0.6066), so no overflow.
#include <mutex>

#include "common.cuh"

namespace {
__device__ int g_chunk_bad = 0;  // a sequence / chunk table out of range (bit 2 of device_error)
constexpr int CL = 16;                       // chunk length
constexpr int KD = RWKV_HD;                  // 64
constexpr int REC = 4 * CL * KD + KD + 2 * CL * CL;  // floats per (chunk, head) record
// record layout (floats): What[CL][KD] | Q[CL][KD] | Bt[CL][KD] | Kt[CL][KD] | gL[KD] | PU[CL][CL] | PY[CL][CL]
constexpr int OFF_W = 0, OFF_Q = CL * KD, OFF_B = 2 * CL * KD, OFF_K = 3 * CL * KD,
              OFF_G = 4 * CL * KD, OFF_PU = 4 * CL * KD + KD, OFF_PY = OFF_PU + CL * CL;
constexpr int RS = KD + 1;  // padded smem row stride (conflict-free column walks)
}  // namespace

// chunk_cu[s] = number of chunks before sequence s (single block, S <= 65536).
__global__ void k_chunk_table(const int* __restrict__ cu, int* __restrict__ chunk_cu, int S) {
  RWKV_GRID_DEP_ENTRY();
  __shared__ int part[1024];
  const int tid = threadIdx.x;
  const int per = (S + blockDim.x - 1) / blockDim.x;
  int local = 0;
  for (int i = tid * per; i < min(S, (tid + 1) * per); ++i) local += (cu[i + 1] - cu[i] + CL - 1) / CL;
  part[tid] = local;
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int i = 0; i < (int)blockDim.x; ++i) {
      const int x = part[i];
      part[i] = run;
      run += x;
    }
  }
  __syncthreads();
  int run = part[tid];
  for (int i = tid * per; i < min(S, (tid + 1) * per); ++i) {
    chunk_cu[i] = run;
    run += (cu[i + 1] - cu[i] + CL - 1) / CL;
  }
  if (tid == (int)blockDim.x - 1) chunk_cu[S] = run;
}

// grid = (max_chunks, H), block = 256. Rows past the sequence end are padded
// with identity transitions (w = 1, a = b = k = r = 0).
__global__ void __launch_bounds__(256) k_chunk_prep(
    const __half* __restrict__ rb, const __half* __restrict__ wb, const __half* __restrict__ kb,
    const __half* __restrict__ ab, const __half* __restrict__ bb, const int* __restrict__ cu,
    const int* __restrict__ chunk_cu, int S, int C, int M, float* __restrict__ rec) {
  RWKV_GRID_DEP_ENTRY();
  __shared__ float sa_[CL * RS], sb_[CL * RS], sk_[CL * RS], sr_[CL * RS], sg[CL * RS];
  __shared__ float Aab[CL][CL + 1], Aak[CL][CL + 1], Brb[CL][CL + 1], Brk[CL][CL + 1],
      Tm[CL][CL + 1], PU[CL][CL + 1];
  __shared__ float Wh[CL * RS];
  __shared__ int info[3];
  const int c = blockIdx.x, h = blockIdx.y, H = gridDim.y, tid = threadIdx.x;
  if (tid == 0) {
    int lo = 0, hi = S;  // find s: chunk_cu[s] <= c < chunk_cu[s+1]
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (chunk_cu[mid] <= c) lo = mid; else hi = mid - 1;
    }
    const int s = lo;
    info[0] = (s < S && c < chunk_cu[S]) ? 1 : 0;
    if (info[0]) {
      const int m0 = cu[s] + (c - chunk_cu[s]) * CL;
      info[1] = m0;
      info[2] = min(CL, cu[s + 1] - m0);
      if (m0 < 0 || info[2] <= 0 || m0 + info[2] > M) {
        atomicExch(&g_chunk_bad, 1);
        info[0] = 0;
      }
    }
  }
  __syncthreads();
  if (!info[0]) return;
  const int m0 = info[1], n = info[2];
  const int hc = h * KD;
  // 1. load (fp16 -> fp32), pad
  for (int i = tid; i < CL * KD; i += 256) {
    const int t = i / KD, k = i % KD;
    float r = 0.f, w = 1.f, kk = 0.f, a = 0.f, b = 0.f;
    if (t < n) {
      const size_t o = (size_t)(m0 + t) * C + hc + k;
      r = h2f(rb[o]); w = h2f(wb[o]); kk = h2f(kb[o]); a = h2f(ab[o]); b = h2f(bb[o]);
    }
    sr_[t * RS + k] = r; sg[t * RS + k] = logf(w); sk_[t * RS + k] = kk; sa_[t * RS + k] = a;
    sb_[t * RS + k] = b;
  }
  __syncthreads();
  // 2. cumulative log decay per column, then decay-scaled vectors
  if (tid < KD) {
    float g = 0.f;
    for (int t = 0; t < CL; ++t) {
      const float gprev = g;
      g += sg[t * RS + tid];
      const float eg = expf(g), egi = expf(-g), egp = expf(gprev);
      sa_[t * RS + tid] *= egp;
      sb_[t * RS + tid] *= egi;
      sk_[t * RS + tid] *= egi;
      sr_[t * RS + tid] *= eg;
      sg[t * RS + tid] = g;
    }
  }
  __syncthreads();
  // 3. the four L x L interaction matrices
  {
    const int t = tid >> 4, j = tid & 15;
    float aab = 0.f, aak = 0.f, brb = 0.f, brk = 0.f;
    if (j <= t) {
      for (int k = 0; k < KD; ++k) {
        const float at = sa_[t * RS + k], rt = sr_[t * RS + k];
        const float bh = sb_[j * RS + k], kh = sk_[j * RS + k];
        aab += at * bh; aak += at * kh; brb += rt * bh; brk += rt * kh;
      }
    }
    Aab[t][j] = (j < t) ? aab : 0.f;
    Aak[t][j] = (j < t) ? aak : 0.f;
    Brb[t][j] = (j <= t) ? brb : 0.f;
    Brk[t][j] = (j <= t) ? brk : 0.f;
  }
  __syncthreads();
  // 4. T = (I - Aab)^{-1}, forward substitution by one warp (lane = column j)
  if (tid < 32) {
    const int j = tid;
    for (int t = 0; t < CL; ++t) {
      if (j < CL) {
        float v = (j == t) ? 1.f : 0.f;
        if (j < t) {
          for (int i = j; i < t; ++i) v += Aab[t][i] * Tm[i][j];
        }
        Tm[t][j] = v;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  float* out = rec + ((size_t)c * H + h) * REC;
  // 5. What = T At (CL x KD), PU = T Aak (CL x CL)
  for (int i = tid; i < CL * KD; i += 256) {
    const int t = i / KD, k = i % KD;
    float v = 0.f;
    for (int q = 0; q <= t; ++q) v += Tm[t][q] * sa_[q * RS + k];
    Wh[t * RS + k] = v;
    out[OFF_W + t * KD + k] = v;
  }
  {
    const int t = tid >> 4, j = tid & 15;
    float v = 0.f;
    for (int q = 0; q <= t; ++q) v += Tm[t][q] * Aak[q][j];
    PU[t][j] = v;
    out[OFF_PU + t * CL + j] = v;
  }
  __syncthreads();
  // 6. Q = Rt + Brb What, PY = Brb PU + Brk, Bt/Kt/gL
  for (int i = tid; i < CL * KD; i += 256) {
    const int t = i / KD, k = i % KD;
    float v = sr_[t * RS + k];
    for (int q = 0; q <= t; ++q) v += Brb[t][q] * Wh[q * RS + k];
    out[OFF_Q + t * KD + k] = v;
    const float gl = expf(sg[(CL - 1) * RS + k]);
    out[OFF_B + t * KD + k] = sb_[t * RS + k] * gl;
    out[OFF_K + t * KD + k] = sk_[t * RS + k] * gl;
    if (t == 0) out[OFF_G + k] = gl;
  }
  {
    const int t = tid >> 4, j = tid & 15;
    float v = Brk[t][j];
    for (int q = 0; q <= t; ++q) v += Brb[t][q] * PU[q][j];
    out[OFF_PY + t * CL + j] = v;
  }
}

// Sum 16 per-lane partials across the warp; lane l ends with the total of index (l >> 1) & 15.
__device__ __forceinline__ float reduce16(float (&p)[16], int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool up = lane & 16;
    const float send = up ? p[i] : p[i + 8];
    const float keep = up ? p[i + 8] : p[i];
    p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool up = lane & 8;
    const float send = up ? p[i] : p[i + 4];
    const float keep = up ? p[i + 4] : p[i];
    p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool up = lane & 4;
    const float send = up ? p[i] : p[i + 2];
    const float keep = up ? p[i + 2] : p[i];
    p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  {
    const bool up = lane & 2;
    const float send = up ? p[0] : p[1];
    const float keep = up ? p[1] : p[0];
    p[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return p[0] + __shfl_xor_sync(0xffffffffu, p[0], 1);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(src));
}

__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, bool pred) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(sz));
}

constexpr int NSTAGE = 4;  // chunk records in flight per CTA
constexpr size_t SCAN_SMEM = (size_t)NSTAGE * (REC + CL * 8 / 2) * sizeof(float);

// grid = (S, H, 8 row groups), block = 256: warp w owns state row v = 8 * group + w.
// Chunk records (and the 16 x 8 values of v the CTA needs) stream through an
// NSTAGE-deep cp.async ring, so each chunk only waits for its own math. y (fp16,
// rounded like the reference's y store) goes to ybuf [M, C].
__global__ void __launch_bounds__(256) k_chunk_scan(
    const __half* __restrict__ vbuf, const float* __restrict__ rec, const int* __restrict__ cu,
    const int* __restrict__ chunk_cu, const int* __restrict__ slots, float* __restrict__ rnn,
    __half* __restrict__ ybuf, int C, int M, int max_chunks, int n_slots) {
  RWKV_GRID_DEP_ENTRY();
  extern __shared__ __align__(16) float scan_smem[];
  float* Rb = scan_smem;                                                   // [NSTAGE][REC]
  __half* Vb = reinterpret_cast<__half*>(scan_smem + (size_t)NSTAGE * REC);  // [NSTAGE][CL][8]
  const int s = blockIdx.x, h = blockIdx.y, H = gridDim.y, grp = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = grp * 8 + warp;
  const int slot = slots ? slots[s] : s;
  const int c0 = chunk_cu[s], c1 = chunk_cu[s + 1];
  const int m_beg = cu[s], m_end = cu[s + 1];
  if (slot < 0 || slot >= n_slots || c0 < 0 || c1 < c0 || c1 > max_chunks || m_beg < 0 ||
      m_end < m_beg || m_end > M || (m_end - m_beg + CL - 1) / CL != c1 - c0) {
    if (tid == 0) atomicExch(&g_chunk_bad, 1);
    return;
  }
  float* Srow = rnn + (((size_t)slot * H + h) * KD + row) * KD;
  float2 st = *reinterpret_cast<const float2*>(Srow + 2 * lane);
  auto stage = [&](int c) {
    if (c < c1) {
      const int buf = (c - c0) % NSTAGE;
      const float* src = rec + ((size_t)c * H + h) * REC;
      for (int i = tid; i < REC / 4; i += 256) cp_async16(Rb + (size_t)buf * REC + 4 * i, src + 4 * i);
      if (tid < CL) {  // token tid's 8 values of v for this CTA's rows (zero past the end)
        const int m = m_beg + (c - c0) * CL + tid;
        const bool ok = m < m_end;
        cp_async16_zfill(Vb + ((size_t)buf * CL + tid) * 8,
                         vbuf + (size_t)(ok ? m : m_beg) * C + h * KD + grp * 8, ok);
      }
    }
    asm volatile("cp.async.commit_group;\n" ::);
  };
#pragma unroll
  for (int i = 0; i < NSTAGE - 1; ++i) stage(c0 + i);
  for (int c = c0; c < c1; ++c) {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(NSTAGE - 2));
    __syncthreads();  // chunk c landed; every warp is done with chunk c - 1's buffer
    stage(c + NSTAGE - 1);
    const int buf = (c - c0) % NSTAGE;
    const float* R = Rb + (size_t)buf * REC;
    const float vt = lane < CL ? __half2float(Vb[((size_t)buf * CL + lane) * 8 + warp]) : 0.f;
    const int m0 = m_beg + (c - c0) * CL;
    const int n = min(CL, m_end - m0);
    float pw[16], pq[16];
#pragma unroll
    for (int t = 0; t < CL; ++t) {
      const float2 w2 = *reinterpret_cast<const float2*>(R + OFF_W + t * KD + 2 * lane);
      const float2 q2 = *reinterpret_cast<const float2*>(R + OFF_Q + t * KD + 2 * lane);
      pw[t] = w2.x * st.x + w2.y * st.y;
      pq[t] = q2.x * st.x + q2.y * st.y;
    }
    // the P_U v / P_Y v terms join the partial sums before the reduction: lane j < 16
    // holds v_j and adds column j of P_U / P_Y to every row's partial
#pragma unroll
    for (int t = 0; t < CL; ++t) {
      if (lane < CL) {
        pw[t] += R[OFF_PU + t * CL + lane] * vt;
        pq[t] += R[OFF_PY + t * CL + lane] * vt;
      }
    }
    const float sa = reduce16(pw, lane);
    const float y = reduce16(pq, lane);
    const int tt = (lane >> 1) & 15;
    if ((lane & 1) == 0 && tt < n) ybuf[(size_t)(m0 + tt) * C + h * KD + row] = f2h(y);
    const float2 gl = *reinterpret_cast<const float2*>(R + OFF_G + 2 * lane);
    float2 n0 = make_float2(st.x * gl.x, st.y * gl.y), n1 = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < CL; j += 2) {
      const float sa0 = __shfl_sync(0xffffffffu, sa, 2 * j);
      const float sa1 = __shfl_sync(0xffffffffu, sa, 2 * j + 2);
      const float v0 = __shfl_sync(0xffffffffu, vt, j);
      const float v1 = __shfl_sync(0xffffffffu, vt, j + 1);
      const float2 b0 = *reinterpret_cast<const float2*>(R + OFF_B + j * KD + 2 * lane);
      const float2 k0 = *reinterpret_cast<const float2*>(R + OFF_K + j * KD + 2 * lane);
      const float2 b1 = *reinterpret_cast<const float2*>(R + OFF_B + (j + 1) * KD + 2 * lane);
      const float2 k1 = *reinterpret_cast<const float2*>(R + OFF_K + (j + 1) * KD + 2 * lane);
      n0.x += sa0 * b0.x + v0 * k0.x;
      n0.y += sa0 * b0.y + v0 * k0.y;
      n1.x += sa1 * b1.x + v1 * k1.x;
      n1.y += sa1 * b1.y + v1 * k1.y;
    }
    st = make_float2(n0.x + n1.x, n0.y + n1.y);
  }
  asm volatile("cp.async.wait_group 0;\n" ::);
  *reinterpret_cast<float2*>(Srow + 2 * lane) = st;
}

// Per-head GroupNorm + bonus + g gate on precomputed y (one warp per head and row).
// grid = M rows, block = C / 2 threads.
template <int SEM>
__global__ void k_wkv_epilogue(const __half* __restrict__ ybuf, const __half* __restrict__ rbuf,
                               const __half* __restrict__ gbuf, size_t plane,
                               const __half* __restrict__ r_k, const __half* __restrict__ lnx_w,
                               const __half* __restrict__ lnx_b, __half* __restrict__ yg, int C) {
  RWKV_GRID_DEP_ENTRY();
  const int m = blockIdx.x, c = threadIdx.x * 2;
  const size_t o = (size_t)m * C + c;
  const float2 y = __half22float2(*reinterpret_cast<const __half2*>(ybuf + o));
  const float mean = warp_sum(y.x + y.y) * (1.0f / RWKV_HD);
  const float dx = y.x - mean, dy = y.y - mean;
  const float var = warp_sum(dx * dx + dy * dy) * (1.0f / RWKV_HD);
  const float rstd = 1.0f / sqrtf(var + 64e-5f);
  const float2 rr = __half22float2(*reinterpret_cast<const __half2*>(rbuf + o));
  const float2 kk = __half22float2(*reinterpret_cast<const __half2*>(gbuf + plane + o));
  const float2 vv = __half22float2(*reinterpret_cast<const __half2*>(gbuf + 2 * plane + o));
  const float2 gg = __half22float2(*reinterpret_cast<const __half2*>(gbuf + 5 * plane + o));
  const float2 rk = __half22float2(*reinterpret_cast<const __half2*>(r_k + c));
  const float2 lw = __half22float2(*reinterpret_cast<const __half2*>(lnx_w + c));
  const float2 lb = __half22float2(*reinterpret_cast<const __half2*>(lnx_b + c));
  float ox, oy;
  if (SEM == SEM_DECODE) {
    float p = rr.x * kk.x * rk.x;
    p += rr.y * kk.y * rk.y;
    const float rkrk = warp_sum(p);
    ox = r16(dx * rstd * lw.x + lb.x + rkrk * vv.x);
    oy = r16(dy * rstd * lw.y + lb.y + rkrk * vv.y);
  } else {
    const float fx = r16(dx * rstd * lw.x + lb.x), fy = r16(dy * rstd * lw.y + lb.y);
    const float rkrk = r16(warp_sum(r16(r16(rr.x * kk.x) * rk.x) + r16(r16(rr.y * kk.y) * rk.y)));
    ox = r16(fx + r16(rkrk * vv.x));
    oy = r16(fy + r16(rkrk * vv.y));
  }
  *reinterpret_cast<__half2*>(yg + o) = __floats2half2_rn(ox * gg.x, oy * gg.y);
}

size_t wkv_chunk_record_bytes(int M, int S, int H) {
  return ((size_t)(M / CL + S) * H * REC) * sizeof(float);
}

// Chunked recurrence only: y (fp16) for every row, state updated in place.
// r..b, y: [M, C] rows (C = H * 64); rnn: [slots, H, 64, 64].
int launch_wkv_chunked(const __half* r, const __half* w, const __half* k, const __half* v,
                       const __half* a, const __half* b, float* rnn, const int* cu,
                       const int* slots, __half* ybuf, float* rec, int* chunk_cu, int M, int S,
                       int H, int n_slots, cudaStream_t st) {
  const int C = H * KD;
  int rc = rwkv_launch("chunk_table", k_chunk_table, dim3(1), dim3(1024), 0, st, cu, chunk_cu, S);
  if (rc) return rc;
  if ((rc = rwkv_launch("chunk_prep", k_chunk_prep, dim3(M / CL + S, H), dim3(256), 0, st, r, w, k,
                        a, b, cu, chunk_cu, S, C, M, rec)))
    return rc;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_chunk_scan, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)SCAN_SMEM);
    if (e != cudaSuccess) {
      rwkv_set_error("chunk_scan: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return RWKV_ERR_CUDA;
    }
    attr_done[dev] = true;
  }
  return rwkv_launch("chunk_scan", k_chunk_scan, dim3(S, H, KD / 8), dim3(256), SCAN_SMEM, st, v,
                     rec, cu, chunk_cu, slots, rnn, ybuf, C, M, M / CL + S, n_slots);
}

int launch_wkv_epilogue(int sem, const __half* ybuf, const __half* rbuf, const __half* gbuf,
                        size_t plane, const __half* r_k, const __half* lnx_w,
                        const __half* lnx_b, __half* yg, int M, int C, cudaStream_t st) {
  return rwkv_launch("wkv_epilogue", sem == SEM_DECODE ? k_wkv_epilogue<SEM_DECODE> : k_wkv_epilogue<SEM_PREFILL>,
                     dim3(M), dim3(C / 2), 0, st, ybuf, rbuf, gbuf, plane, r_k, lnx_w, lnx_b, yg, C);
}

__global__ void k_uniform_cu(int* cu, int S, int T) {
  RWKV_GRID_DEP_ENTRY();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i <= S) cu[i] = i * T;
}

int wkv_chunk_bad_flag() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_chunk_bad, sizeof(int));
  if (v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_chunk_bad, &z, sizeof(int));
  }
  return v;
}

extern "C" size_t rwkv7_dplr_chunked_workspace_bytes(int n_seq, int T, int H) {
  if (n_seq <= 0 || T <= 0 || H <= 0) return 0;
  const size_t cu = ((size_t)(n_seq + 1) * 2 * sizeof(int) + 255) & ~size_t(255);
  return cu + wkv_chunk_record_bytes(n_seq * T, n_seq, H);
}

extern "C" int rwkv7_dplr_chunked(void* S, const void* r, const void* w, const void* k,
                                  const void* v, const void* a, const void* b, void* y, int n_seq,
                                  int T, int H, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  rwkv_chain_begin();
  if (!S || !r || !w || !k || !v || !a || !b || !y || n_seq <= 0 || T <= 0 || H <= 0) {
    rwkv_set_error("rwkv7_dplr_chunked: null pointer or bad size (n_seq=%d, T=%d, H=%d)", n_seq,
                   T, H);
    return RWKV_ERR_ARG;
  }
  const size_t need = rwkv7_dplr_chunked_workspace_bytes(n_seq, T, H);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) {
    rwkv_set_error("rwkv7_dplr_chunked: workspace needs %zu bytes, 256-aligned (got %zu)", need,
                   workspace_bytes);
    return RWKV_ERR_SPACE;
  }
  if ((size_t)n_seq * T * H * KD > ((size_t)1 << 31)) {
    rwkv_set_error("rwkv7_dplr_chunked: problem too large (%d x %d x %d)", n_seq, T, H);
    return RWKV_ERR_ARG;
  }
  cudaStream_t st = (cudaStream_t)stream;
  int* cu = static_cast<int*>(workspace);
  int* chunk_cu = cu + n_seq + 1;
  float* rec = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                        (((size_t)(n_seq + 1) * 2 * sizeof(int) + 255) & ~size_t(255)));
  int rc = rwkv_launch("uniform_cu", k_uniform_cu, dim3((n_seq + 256) / 256), dim3(256), 0, st, cu,
                       n_seq, T);
  if (rc) return rc;
  return launch_wkv_chunked((const __half*)r, (const __half*)w, (const __half*)k,
                            (const __half*)v, (const __half*)a, (const __half*)b, (float*)S, cu,
                            nullptr, (__half*)y, rec, chunk_cu, n_seq * T, n_seq, H, n_seq, st);
}

// ---------------------------------------------------------------------------
// rwkv7_dplr_chunked without a caller-provided workspace.
//
// Some callers cannot allocate device memory at the point where they run the
// recurrence: code running inside an allocator-free region (a memory pool
// that must not grow, a host framework that owns all device allocations and
// only hands out input/output buffers, a plugin loaded into a process whose
// allocator is not reachable from this library). For them the scratch lives
// in this file-scope array instead: every GPU that loads the library holds
// these 16 MiB until the process exits. In host code `g_noalloc_scratch` is
// only a host-side stand-in for the symbol, never a device address; the device
// address comes from cudaGetSymbolAddress, once per device, on that device's
// first call (make that first call before any stream capture).
namespace {
constexpr size_t NOALLOC_BYTES = (size_t)16 << 20;
}
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_BYTES];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64] = {};

extern "C" int rwkv7_dplr_chunked_noalloc(void* S, const void* r, const void* w, const void* k,
                                          const void* v, const void* a, const void* b, void* y,
                                          int n_seq, int T, int H, void* stream) {
  rwkv_chain_begin();
  if (n_seq <= 0 || T <= 0 || H <= 0) {
    rwkv_set_error("rwkv7_dplr_chunked_noalloc: bad size (n_seq=%d, T=%d, H=%d)", n_seq, T, H);
    return RWKV_ERR_ARG;
  }
  const size_t need = rwkv7_dplr_chunked_workspace_bytes(n_seq, T, H);
  if (need > NOALLOC_BYTES) {
    rwkv_set_error(
        "rwkv7_dplr_chunked_noalloc: n_seq=%d T=%d H=%d needs %zu bytes of scratch, more than the "
        "built-in %zu; use rwkv7_dplr_chunked with a workspace",
        n_seq, T, H, need, NOALLOC_BYTES);
    return RWKV_ERR_SPACE;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    rwkv_set_error("rwkv7_dplr_chunked_noalloc: no usable current device");
    return RWKV_ERR_CUDA;
  }
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      cudaError_t e = cudaGetSymbolAddress(&g_noalloc_ptr[dev], g_noalloc_scratch);
      if (e != cudaSuccess) {
        g_noalloc_ptr[dev] = nullptr;
        rwkv_set_error("rwkv7_dplr_chunked_noalloc: cudaGetSymbolAddress failed: %s",
                       cudaGetErrorString(e));
        return RWKV_ERR_CUDA;
      }
    }
    ptr = g_noalloc_ptr[dev];
  }
  // Nothing in the scratch has to start at zero: the sequence offsets, the
  // chunk table and every chunk record read later are written first by this call.
  return rwkv7_dplr_chunked(S, r, w, k, v, a, b, y, n_seq, T, H, ptr, NOALLOC_BYTES, stream);
}
