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
__device__ int g_chunk_bad = 0;  // 1: a sequence / chunk table out of range; 2: a scan wait gave up
constexpr int CL = 16;                       // chunk length
constexpr int KD = RWKV_HD;                  // 64
constexpr int RWS = 2 * CL + KD;             // per-row floats: PU v | PY v | U
constexpr int SHARED_F = 3 * CL * KD + KD;    // row-independent part of a record
constexpr int REC = SHARED_F + KD * RWS;      // floats per (chunk, head) record
// record layout (floats): What[CL][KD] | Q[CL][KD] | Bt[CL][KD] | gL[KD] |
//   per state row v: (PU v)[CL] | (PY v)[CL] | U[KD]   (the value-dependent terms, [KD][RWS])
// with U = sum_j v_j Kt_j, the whole value input of the chunk to that state row.
constexpr int OFF_W = 0, OFF_Q = CL * KD, OFF_B = 2 * CL * KD, OFF_G = 3 * CL * KD,
              OFF_RW = SHARED_F;
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
__global__ void __launch_bounds__(256, 4) k_chunk_prep(
    const __half* __restrict__ rb, const __half* __restrict__ wb, const __half* __restrict__ kb,
    const __half* __restrict__ vb, const __half* __restrict__ ab, const __half* __restrict__ bb,
    const int* __restrict__ cu,
    const int* __restrict__ chunk_cu, int S, int C, int M, float* __restrict__ rec) {
  RWKV_GRID_DEP_ENTRY();
  __shared__ float sa_[CL * RS], sb_[CL * RS], sk_[CL * RS], sr_[CL * RS], sg[CL * RS];
  __shared__ float Aab[CL][CL + 1], Aak[CL][CL + 1], Brb[CL][CL + 1], Brk[CL][CL + 1],
      Tm[CL][CL + 1], PU[CL][CL + 1], PY[CL][CL + 1];
  __shared__ float sv_[CL * RS];
  __shared__ float glv[KD];  // e^{G_L}: the chunk's total decay per key column
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
  // 1. load (fp16 -> fp32, two channels per thread), pad
  for (int i = tid; i < CL * KD / 2; i += 256) {
    const int t = i / (KD / 2), k = 2 * (i % (KD / 2));
    float2 r = make_float2(0.f, 0.f), w = make_float2(1.f, 1.f), kk = r, vv = r, a = r, b = r;
    if (t < n) {
      const size_t o = (size_t)(m0 + t) * C + hc + k;
      auto ld = [&](const __half* p) { return __half22float2(*reinterpret_cast<const __half2*>(p + o)); };
      r = ld(rb); w = ld(wb); kk = ld(kb); vv = ld(vb); a = ld(ab); b = ld(bb);
    }
    const int q = t * RS + k;
    sv_[q] = vv.x; sv_[q + 1] = vv.y;
    sr_[q] = r.x; sr_[q + 1] = r.y;
    sg[q] = logf(w.x); sg[q + 1] = logf(w.y);
    sk_[q] = kk.x; sk_[q + 1] = kk.y;
    sa_[q] = a.x; sa_[q + 1] = a.y;
    sb_[q] = b.x; sb_[q + 1] = b.y;
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
    glv[tid] = expf(g);
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
  }
  __syncthreads();
  // 6. Q = Rt + Brb What, PY = Brb PU + Brk, Bt/Kt/gL
  for (int i = tid; i < CL * KD; i += 256) {
    const int t = i / KD, k = i % KD;
    float v = sr_[t * RS + k];
    for (int q = 0; q <= t; ++q) v += Brb[t][q] * Wh[q * RS + k];
    out[OFF_Q + t * KD + k] = v;
    const float gl = glv[k];
    out[OFF_B + t * KD + k] = sb_[t * RS + k] * gl;
    if (t == 0) out[OFF_G + k] = gl;
  }
  {
    const int t = tid >> 4, j = tid & 15;
    float v = Brk[t][j];
    for (int q = 0; q <= t; ++q) v += Brb[t][q] * PU[q][j];
    PY[t][j] = v;
  }
  __syncthreads();
  // 7. the value-dependent terms per state row: (PU v)_t, (PY v)_t and U = sum_j v_j Kt_j,
  // register-blocked over 4 state rows per thread
  {
    const int t = tid & 15, r0 = (tid >> 4) * 4;
    float pu[4] = {}, py[4] = {};
#pragma unroll 4
    for (int j = 0; j < CL; ++j) {
      const float a = PU[t][j], b = PY[t][j];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float vj = sv_[j * RS + r0 + r];
        pu[r] += a * vj;
        py[r] += b * vj;
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float* o = out + OFF_RW + (r0 + r) * RWS;
      o[t] = pu[r];
      o[CL + t] = py[r];
    }
  }
  {
    const int k0 = (tid & 15) * 4, r0 = (tid >> 4) * 4;
    float u[4][4] = {};
#pragma unroll 2
    for (int j = 0; j < CL; ++j) {
      float vv[4], kk[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        vv[e] = sv_[j * RS + r0 + e];
        kk[e] = sk_[j * RS + k0 + e];
      }
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) u[r][c] += vv[r] * kk[c];
    }
    const float4 g4 = make_float4(glv[k0], glv[k0 + 1], glv[k0 + 2], glv[k0 + 3]);
#pragma unroll
    for (int r = 0; r < 4; ++r)
      *reinterpret_cast<float4*>(out + OFF_RW + (r0 + r) * RWS + 2 * CL + k0) =
          make_float4(u[r][0] * g4.x, u[r][1] * g4.y, u[r][2] * g4.z, u[r][3] * g4.w);
  }
}

// ---- chunk scan: bounded mbarrier waits and 1-D bulk copies ------------------------
namespace {
constexpr uint64_t SCAN_WAIT_NS = 200ull * 1000 * 1000;  // 200 ms: a bounded wait gave up
__device__ __forceinline__ uint32_t sm_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void sc_mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sm_addr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void sc_mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sm_addr(b)) : "memory");
}
__device__ __forceinline__ void sc_mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sm_addr(b)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool sc_mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(sm_addr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for phase `parity` of b for at most SCAN_WAIT_NS; false (and the error flag) on expiry.
__device__ __forceinline__ bool sc_mbar_wait(uint64_t* b, uint32_t parity) {
  if (sc_mbar_try(b, parity)) return true;
  const uint64_t t0 = gtimer();
  while (!sc_mbar_try(b, parity)) {
    if (gtimer() - t0 > SCAN_WAIT_NS) {
      atomicOr(&g_chunk_bad, 2);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void sc_bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                            uint64_t* b) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          sm_addr(dst)),
      "l"(src), "r"(bytes), "r"(sm_addr(b))
      : "memory");
}

// 4-wide dot product with packed fp32 pairs.
__device__ __forceinline__ float dot4(float4 a, float2 s01, float2 s23) {
  const float2 p = __ffma2_rn(make_float2(a.z, a.w), s23, __fmul2_rn(make_float2(a.x, a.y), s01));
  return p.x + p.y;
}

constexpr int SCAN_ROWS = 8;                        // state rows per CTA
constexpr int SCAN_THREADS = 128;                   // four warps, two rows each
constexpr int SLICE_F = SCAN_ROWS * RWS;            // per-CTA part of a record's row terms
constexpr int STAGE_F = SHARED_F + SLICE_F;         // floats per ring stage
// Chunk records in flight per CTA. Eight stages (125 KB) also keep a second scan CTA
// off the SM: placed early by programmatic dependent launch, CTAs could otherwise
// pile up two or three per SM, and the slowest SM sets the scan's time.
constexpr int NSTAGE = 8;
constexpr size_t SCAN_SMEM = (size_t)NSTAGE * STAGE_F * sizeof(float) + 2 * NSTAGE * sizeof(uint64_t);
static_assert((SHARED_F * 4) % 16 == 0 && (SLICE_F * 4) % 16 == 0 && (REC * 4) % 16 == 0,
              "bulk copies need 16-byte multiples");
static_assert(SCAN_SMEM > 114 * 1024 && SCAN_SMEM <= 227 * 1024, "one scan CTA per SM");
}  // namespace

// grid = (S, H, KD / 8 row groups), block = 128. Each half-warp owns one state row
// (lane l of the half holds keys 4l..4l+3 of it), so a warp carries two rows. Chunk
// records stream through an NSTAGE ring of 1-D bulk copies (mbarrier full / empty).
// Per chunk a half-warp forms the 16 What and 16 Q dot products of its row, reduces
// the 32 partial sums across its 16 lanes (lane l ends with sums 2l and 2l + 1: the
// in-chunk states sa for l < 8, the outputs y for l >= 8), adds the value terms
// PU v / PY v that k_chunk_prep precomputed, writes y (fp16, rounded like the
// reference's y store) to ybuf [M, C] and advances the fp32 state by
//   s <- s * gL + sum_j sa_j Bt_j + U.
__global__ void __launch_bounds__(SCAN_THREADS) k_chunk_scan(
    const float* __restrict__ rec, const int* __restrict__ cu, const int* __restrict__ chunk_cu,
    const int* __restrict__ slots, float* __restrict__ rnn, __half* __restrict__ ybuf, int C,
    int M, int max_chunks, int n_slots) {
  RWKV_GRID_DEP_ENTRY();
  extern __shared__ __align__(128) float scan_smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(scan_smem + (size_t)NSTAGE * STAGE_F);
  uint64_t* empty = full + NSTAGE;
  const int s = blockIdx.x, h = blockIdx.y, H = gridDim.y, grp = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hl = lane & 15, lrow = warp * 2 + (lane >> 4);
  const int row = grp * SCAN_ROWS + lrow;
  const int slot = slots ? slots[s] : s;
  const int c0 = chunk_cu[s], c1 = chunk_cu[s + 1];
  const int m_beg = cu[s], m_end = cu[s + 1];
  if (slot < 0 || slot >= n_slots || c0 < 0 || c1 < c0 || c1 > max_chunks || m_beg < 0 ||
      m_end < m_beg || m_end > M || (m_end - m_beg + CL - 1) / CL != c1 - c0) {
    if (tid == 0) atomicOr(&g_chunk_bad, 1);
    return;
  }
  if (tid == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      sc_mbar_init(&full[i], 1);
      sc_mbar_init(&empty[i], SCAN_THREADS / 32);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  float* Srow = rnn + (((size_t)slot * H + h) * KD + row) * KD + 4 * hl;
  float4 st = *reinterpret_cast<const float4*>(Srow);
  int issued = 0;  // chunks whose copies thread 0 has issued
  auto issue = [&](int c) {
    const int buf = (c - c0) % NSTAGE;
    float* dst = scan_smem + (size_t)buf * STAGE_F;
    const float* src = rec + ((size_t)c * H + h) * REC;
    sc_mbar_expect_tx(&full[buf], STAGE_F * 4);
    sc_bulk_g2s(dst, src, SHARED_F * 4, &full[buf]);
    sc_bulk_g2s(dst + SHARED_F, src + OFF_RW + grp * SLICE_F, SLICE_F * 4, &full[buf]);
    ++issued;
  };
  if (tid == 0)
    for (int i = 0; i < NSTAGE && c0 + i < c1; ++i) issue(c0 + i);
  bool ok = true;
  for (int c = c0; c < c1; ++c) {
    const int it = c - c0, buf = it % NSTAGE;
    // refill the stage chunk c - 1 used, once all four warps are done with it
    if (tid == 0 && it >= 1 && c - 1 + NSTAGE < c1) {
      if (sc_mbar_wait(&empty[(it - 1) % NSTAGE], ((it - 1) / NSTAGE) & 1)) issue(c - 1 + NSTAGE);
      else ok = false;
    }
    ok = __all_sync(0xffffffffu, ok && sc_mbar_wait(&full[buf], (it / NSTAGE) & 1));
    if (!ok) break;
    const float* R = scan_smem + (size_t)buf * STAGE_F;
    const float* RW = R + SHARED_F + lrow * RWS;
    const float2 s01 = make_float2(st.x, st.y), s23 = make_float2(st.z, st.w);
    float p[32];
#pragma unroll
    for (int t = 0; t < CL; ++t) {
      p[t] = dot4(*reinterpret_cast<const float4*>(R + OFF_W + t * KD + 4 * hl), s01, s23);
      p[CL + t] = dot4(*reinterpret_cast<const float4*>(R + OFF_Q + t * KD + 4 * hl), s01, s23);
    }
    // transpose-reduce over the 16 lanes of the half-warp: 32 -> 16 -> 8 -> 4 -> 2 sums
#pragma unroll
    for (int m = 8, half = 16; m >= 1; m >>= 1, half >>= 1) {
      const bool up = lane & m;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = up ? p[i] : p[i + half];
        const float keep = up ? p[i + half] : p[i];
        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
      }
    }
    // lane hl holds sums 2hl, 2hl + 1: (What s)_t for hl < 8, (Q s)_t for hl >= 8, t = 2hl mod 16
    const float2 add = *reinterpret_cast<const float2*>(RW + 2 * hl);
    const float o0 = p[0] + add.x, o1 = p[1] + add.y;
    if (hl >= 8) {
      const int m0 = m_beg + it * CL + 2 * hl - CL;
      __half* yp = ybuf + (size_t)m0 * C + h * KD + row;
      if (m0 < m_end) yp[0] = f2h(o0);
      if (m0 + 1 < m_end) yp[C] = f2h(o1);
    }
    const float4 gl = *reinterpret_cast<const float4*>(R + OFF_G + 4 * hl);
    const float4 u = *reinterpret_cast<const float4*>(RW + 2 * CL + 4 * hl);
    float2 n01 = __ffma2_rn(s01, make_float2(gl.x, gl.y), make_float2(u.x, u.y));
    float2 n23 = __ffma2_rn(s23, make_float2(gl.z, gl.w), make_float2(u.z, u.w));
    float2 m01 = make_float2(0.f, 0.f), m23 = make_float2(0.f, 0.f);
    const int src = lane & 16;
#pragma unroll
    for (int j = 0; j < CL; ++j) {
      const float sa = __shfl_sync(0xffffffffu, (j & 1) ? o1 : o0, src + (j >> 1));
      const float4 b = *reinterpret_cast<const float4*>(R + OFF_B + j * KD + 4 * hl);
      const float2 sa2 = make_float2(sa, sa);
      if (j & 1) {
        m01 = __ffma2_rn(sa2, make_float2(b.x, b.y), m01);
        m23 = __ffma2_rn(sa2, make_float2(b.z, b.w), m23);
      } else {
        n01 = __ffma2_rn(sa2, make_float2(b.x, b.y), n01);
        n23 = __ffma2_rn(sa2, make_float2(b.z, b.w), n23);
      }
    }
    n01 = __fadd2_rn(n01, m01);
    n23 = __fadd2_rn(n23, m23);
    st = make_float4(n01.x, n01.y, n23.x, n23.y);
    __syncwarp();
    if (lane == 0) sc_mbar_arrive(&empty[buf]);
  }
  if (!ok) {
    // leave no bulk copy in flight into this CTA's shared memory
    if (tid == 0)
      for (int i = 0; i < NSTAGE && issued > 0; ++i) {
        const int c = c0 + issued - 1 - i;
        if (c < c0) break;
        const int k = c - c0;
        sc_mbar_wait(&full[k % NSTAGE], (k / NSTAGE) & 1);
      }
    return;
  }
  *reinterpret_cast<float4*>(Srow) = st;
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
// chunk_cu[s] = chunks before sequence s; depends on the sequence table only, so a
// forward computes it once for all layers.
int launch_chunk_table(const int* cu, int* chunk_cu, int S, cudaStream_t st) {
  return rwkv_launch("chunk_table", k_chunk_table, dim3(1), dim3(1024), 0, st, cu, chunk_cu, S);
}

// Chunk transforms + scan of one layer; `chunk_cu` must already hold the chunk table.
int launch_wkv_chunked(const __half* r, const __half* w, const __half* k, const __half* v,
                       const __half* a, const __half* b, float* rnn, const int* cu,
                       const int* slots, __half* ybuf, float* rec, int* chunk_cu, int M, int S,
                       int H, int n_slots, cudaStream_t st) {
  const int C = H * KD;
  int rc;
  if ((rc = rwkv_launch("chunk_prep", k_chunk_prep, dim3(M / CL + S, H), dim3(256), 0, st, r, w, k,
                        v, a, b, cu, chunk_cu, S, C, M, rec)))
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
  return rwkv_launch("chunk_scan", k_chunk_scan, dim3(S, H, KD / SCAN_ROWS), dim3(SCAN_THREADS), SCAN_SMEM,
                     st, rec, cu, chunk_cu, slots, rnn, ybuf, C, M, M / CL + S, n_slots);
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
  if (reinterpret_cast<uintptr_t>(S) & 15) {
    rwkv_set_error("rwkv7_dplr_chunked: S must be 16-byte aligned");
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
  if ((rc = launch_chunk_table(cu, chunk_cu, n_seq, st))) return rc;
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
// these 32 MiB until the process exits. In host code `g_noalloc_scratch` is
// only a host-side stand-in for the symbol, never a device address; the device
// address comes from cudaGetSymbolAddress, once per device, on that device's
// first call (make that first call before any stream capture).
namespace {
constexpr size_t NOALLOC_BYTES = (size_t)32 << 20;
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
