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
#include <climits>
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace {
__device__ int g_chunk_bad = 0;  // 1: a sequence / chunk table out of range; 2: a scan wait gave up
constexpr int CL = 16;                       // chunk length
constexpr int KD = RWKV_HD;                  // 64
#ifndef RWS_PAD
#define RWS_PAD 4  // 400-byte rows: consecutive rows' 16-byte loads fall on distinct banks
#endif
constexpr int RWS = 2 * CL + KD + RWS_PAD;   // per-row floats: PU v | PY v | U | pad
constexpr int SHARED_F = 3 * CL * KD + KD;    // row-independent part of a record
constexpr int REC = SHARED_F + KD * RWS;      // floats per (chunk, head) record
// record layout (floats): What[CL][KD] | Q[CL][KD] | Bt[CL][KD] | gL[KD] |
//   per state row v: (PU v)[CL] | (PY v)[CL] | U[KD]   (the value-dependent terms, [KD][RWS])
// with U = sum_j v_j Kt_j, the whole value input of the chunk to that state row.
constexpr int OFF_W = 0, OFF_Q = CL * KD, OFF_B = 2 * CL * KD, OFF_G = 3 * CL * KD,
              OFF_RW = SHARED_F;
// Shared-memory row strides of the chunk prep. Rows read along k or by broadcast use
// KD (float4 rows); sb_ / sk_, which 16 threads read at 16 different rows at once, use
// KD + 4 so that a quarter-warp's float4 loads fall in distinct banks.
constexpr int RSA = KD, RSB = KD + 4;
#ifndef PREP_MINB
#define PREP_MINB 7
#endif
// Two-level scan: a sequence's chunks are cut into segments of SEG chunks (128 tokens).
// Segments are scanned concurrently (the first from the true state, the others from
// zero); each segment's transfer matrix Phi (product of its chunk maps) then carries
// the true state across segments, and Q Phi corrects the later segments' outputs.
#ifndef SEG_CHUNKS
#define SEG_CHUNKS 8  // measured at T=4096: 8 beats 16 (0.5 %) and 32 (-5 %)
#endif
constexpr int SEG = SEG_CHUNKS;
// chunks of a segment corrected by one k_seg_fix CTA (a divisor of SEG)
#ifndef FIX_CHUNKS
#define FIX_CHUNKS 4  // measured at T=4096: 4 beats 8 (one CTA per segment) by 0.5 %, 2 and 1
#endif
static_assert(SEG % FIX_CHUNKS == 0, "FIX_CHUNKS must divide SEG_CHUNKS");
}  // namespace

// chunk_cu[s] = chunks before sequence s, seg_cu[s] = segments (SEG chunks each) before
// sequence s (single block, S <= 65536).
__global__ void k_chunk_table(const int* __restrict__ cu, int* __restrict__ chunk_cu,
                              int* __restrict__ seg_cu, int S) {
  RWKV_GRID_DEP_ENTRY();
  __shared__ int part[2][1024];
  const int tid = threadIdx.x;
  const int per = (S + blockDim.x - 1) / blockDim.x;
  int lc = 0, ls = 0;
  for (int i = tid * per; i < min(S, (tid + 1) * per); ++i) {
    const int n = (cu[i + 1] - cu[i] + CL - 1) / CL;
    lc += n;
    ls += (n + SEG - 1) / SEG;
  }
  part[0][tid] = lc;
  part[1][tid] = ls;
  __syncthreads();
  if (tid < 2) {
    int run = 0;
    for (int i = 0; i < (int)blockDim.x; ++i) {
      const int x = part[tid][i];
      part[tid][i] = run;
      run += x;
    }
  }
  __syncthreads();
  int rc = part[0][tid], rs = part[1][tid];
  for (int i = tid * per; i < min(S, (tid + 1) * per); ++i) {
    chunk_cu[i] = rc;
    seg_cu[i] = rs;
    const int n = (cu[i + 1] - cu[i] + CL - 1) / CL;
    rc += n;
    rs += (n + SEG - 1) / SEG;
  }
  if (tid == (int)blockDim.x - 1) {
    chunk_cu[S] = rc;
    seg_cu[S] = rs;
  }
}

// Largest s in [0, S) with tab[s] <= x (tab non-decreasing, tab[0] = 0).
__device__ __forceinline__ int seq_of(const int* tab, int S, int x) {
  int lo = 0, hi = S - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tab[mid] <= x) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// grid = (max_chunks, H), block = 256. Rows past the sequence end are padded
// with identity transitions (w = 1, a = b = k = r = 0).
__global__ void __launch_bounds__(256, PREP_MINB) k_chunk_prep(
    const __half* __restrict__ rb, const __half* __restrict__ wb, const __half* __restrict__ kb,
    const __half* __restrict__ vb, const __half* __restrict__ ab, const __half* __restrict__ bb,
    const int* __restrict__ cu,
    const int* __restrict__ chunk_cu, int S, int C, int M, float* __restrict__ rec) {
  RWKV_GRID_DEP_ENTRY();
  __shared__ __align__(16) float sa_[CL * RSA], sb_[CL * RSB], sk_[CL * RSB], sr_[CL * RSA],
      sg[CL * RSA];
  __shared__ float Aab[CL][CL + 1], Aak[CL][CL + 1], Brb[CL][CL + 1], Brk[CL][CL + 1],
      Tm[CL][CL + 1];
  __shared__ __align__(16) float sv_[CL * RSA];
  __shared__ __align__(16) float glv[KD];  // e^{G_L}: the chunk's total decay per key column
  // storage reused once its first tenant is dead (keeps the CTA small: 7 per SM):
  float* Wh = sg;           // What, written in step 5; sg is last read in step 2
  float(*PU)[CL + 1] = Aab;  // P_U, written in step 5; A_ab is last read in step 4
  float(*PY)[CL + 1] = Brk;  // P_Y = B_rk + B_rb P_U, written in place over B_rk
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
    const int q = t * RSA + k, qb = t * RSB + k;
    sv_[q] = vv.x; sv_[q + 1] = vv.y;
    sr_[q] = r.x; sr_[q + 1] = r.y;
    sg[q] = logf(w.x); sg[q + 1] = logf(w.y);
    sk_[qb] = kk.x; sk_[qb + 1] = kk.y;
    sa_[q] = a.x; sa_[q + 1] = a.y;
    sb_[qb] = b.x; sb_[qb + 1] = b.y;
  }
  __syncthreads();
  // 2. cumulative log decay per column (summed in t order by one thread per column), then
  // the decay-scaled vectors by all threads (column k, rows 4 tq .. 4 tq + 3)
  if (tid < KD) {
    float lw[CL];
#pragma unroll
    for (int t = 0; t < CL; ++t) lw[t] = sg[t * RSA + tid];
    float g = 0.f;
#pragma unroll
    for (int t = 0; t < CL; ++t) {
      g += lw[t];
      sg[t * RSA + tid] = g;
    }
  }
  __syncthreads();
  {
    const int k = tid & (KD - 1), tq = tid / KD;
    float egp = tq ? expf(sg[(4 * tq - 1) * RSA + k]) : 1.f;  // e^{G_{t-1}}
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = 4 * tq + i;
      const float eg = expf(sg[t * RSA + k]), egi = 1.0f / eg;
      sa_[t * RSA + k] *= egp;
      sb_[t * RSB + k] *= egi;
      sk_[t * RSB + k] *= egi;
      sr_[t * RSA + k] *= eg;
      egp = eg;
    }
    if (tq == CL / 4 - 1) glv[k] = egp;  // e^{G_L}
  }
  __syncthreads();
  // 3. the four L x L interaction matrices
  {
    const int t = tid >> 4, j = tid & 15;
    float aab = 0.f, aak = 0.f, brb = 0.f, brk = 0.f;
    if (j <= t) {
      // float4 rows, each sum still taken in k order
      const float4* A4 = reinterpret_cast<const float4*>(sa_ + t * RSA);
      const float4* R4 = reinterpret_cast<const float4*>(sr_ + t * RSA);
      const float4* B4 = reinterpret_cast<const float4*>(sb_ + j * RSB);
      const float4* K4 = reinterpret_cast<const float4*>(sk_ + j * RSB);
      for (int k4 = 0; k4 < KD / 4; ++k4) {
        const float4 at = A4[k4], rt = R4[k4], bh = B4[k4], kh = K4[k4];
        aab += at.x * bh.x; aak += at.x * kh.x; brb += rt.x * bh.x; brk += rt.x * kh.x;
        aab += at.y * bh.y; aak += at.y * kh.y; brb += rt.y * bh.y; brk += rt.y * kh.y;
        aab += at.z * bh.z; aak += at.z * kh.z; brb += rt.z * bh.z; brk += rt.z * kh.z;
        aab += at.w * bh.w; aak += at.w * kh.w; brb += rt.w * bh.w; brk += rt.w * kh.w;
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
  // 5. What = T At (CL x KD), PU = T Aak (CL x CL). Triangular rows are paired: warp w
  // computes rows w and CL - 1 - w (two columns per lane), 17 row steps for every warp.
  const int wp = tid >> 5, k2 = (tid & 31) * 2;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int t = half ? CL - 1 - wp : wp;
    float2 v = make_float2(0.f, 0.f);
    for (int q = 0; q <= t; ++q) {
      const float tm = Tm[t][q];
      const float2 a = *reinterpret_cast<const float2*>(sa_ + q * RSA + k2);
      v.x += tm * a.x; v.y += tm * a.y;
    }
    *reinterpret_cast<float2*>(Wh + t * RSA + k2) = v;
    *reinterpret_cast<float2*>(out + OFF_W + t * KD + k2) = v;
  }
  {
    const int t = tid >> 4, j = tid & 15;
    float v = 0.f;
    for (int q = 0; q <= t; ++q) v += Tm[t][q] * Aak[q][j];
    PU[t][j] = v;
  }
  __syncthreads();
  // 6. Q = Rt + Brb What, PY = Brb PU + Brk, Bt/Kt/gL (rows paired as in step 5)
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int t = half ? CL - 1 - wp : wp;
    float2 v = *reinterpret_cast<const float2*>(sr_ + t * RSA + k2);
    for (int q = 0; q <= t; ++q) {
      const float b = Brb[t][q];
      const float2 w2 = *reinterpret_cast<const float2*>(Wh + q * RSA + k2);
      v.x += b * w2.x; v.y += b * w2.y;
    }
    *reinterpret_cast<float2*>(out + OFF_Q + t * KD + k2) = v;
    const float2 gl = *reinterpret_cast<const float2*>(glv + k2);
    const float2 bt = *reinterpret_cast<const float2*>(sb_ + t * RSB + k2);
    *reinterpret_cast<float2*>(out + OFF_B + t * KD + k2) = make_float2(bt.x * gl.x, bt.y * gl.y);
    if (t == 0) *reinterpret_cast<float2*>(out + OFF_G + k2) = gl;
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
      const float4 v4 = *reinterpret_cast<const float4*>(sv_ + j * RSA + r0);
      const float vj[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        pu[r] += a * vj[r];
        py[r] += b * vj[r];
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
      const float4 v4 = *reinterpret_cast<const float4*>(sv_ + j * RSA + r0);
      const float4 k4 = *reinterpret_cast<const float4*>(sk_ + j * RSB + k0);
      const float vv[4] = {v4.x, v4.y, v4.z, v4.w}, kk[4] = {k4.x, k4.y, k4.z, k4.w};
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

constexpr int SCAN_ROWS = 32;                       // state rows per CTA
constexpr int SCAN_THREADS = 256;                   // eight warps, four rows each
constexpr int SLICE_F = SCAN_ROWS * RWS;            // per-CTA part of a record's row terms
constexpr int STAGE_F = SHARED_F + SLICE_F;         // floats per ring stage
// Chunk records in flight per CTA: a segment has at most SEG chunks and three
// segment CTAs share an SM, so a two-stage ring (50 KB) suffices; measured at
// T=4096, two stages beat three (0.6 %: more of the SM's memory left to L1).
#ifndef SCAN_NSTAGE
#define SCAN_NSTAGE 2
#endif
constexpr int NSTAGE = SCAN_NSTAGE;
constexpr size_t SCAN_SMEM = (size_t)NSTAGE * STAGE_F * sizeof(float) + 2 * NSTAGE * sizeof(uint64_t);
static_assert((SHARED_F * 4) % 16 == 0 && (SLICE_F * 4) % 16 == 0 && (REC * 4) % 16 == 0,
              "bulk copies need 16-byte multiples");
}  // namespace

// grid = (max segments, H, KD / 8 row groups), block = 128: one segment of one
// sequence per CTA (segment 0 starts from the sequence's state in rnn and writes final
// fp16 outputs; later segments start from zero and write fp32 outputs to yf32 and
// their end state to lbuf, for k_seg_combine / k_seg_fix). Each half-warp owns one state row
// (lane l of the half holds keys 4l..4l+3 of it), so a warp carries two rows. Chunk
// records stream through an NSTAGE ring of 1-D bulk copies (mbarrier full / empty).
// Per chunk a half-warp forms the 16 What and 16 Q dot products of its row, reduces
// the 32 partial sums across its 16 lanes (lane l ends with sums 2l and 2l + 1: the
// in-chunk states sa for l < 8, the outputs y for l >= 8), adds the value terms
// PU v / PY v that k_chunk_prep precomputed, writes y (fp16, rounded like the
// reference's y store) to ybuf [M, C] and advances the fp32 state by
//   s <- s * gL + sum_j sa_j Bt_j + U.
__device__ __forceinline__ void chunk_scan_body(
    int gs, int h, int H, int grp, float* scan_smem,
    const float* __restrict__ rec, const int* __restrict__ cu, const int* __restrict__ chunk_cu,
    const int* __restrict__ seg_cu, const int* __restrict__ slots, float* __restrict__ rnn,
    __half* __restrict__ ybuf, float* __restrict__ yf32, float* __restrict__ lbuf, int S, int C,
    int M, int max_chunks, int n_slots) {
  uint64_t* full = reinterpret_cast<uint64_t*>(scan_smem + (size_t)NSTAGE * STAGE_F);
  uint64_t* empty = full + NSTAGE;
  if (gs >= seg_cu[S]) return;
  const int s = seq_of(seg_cu, S, gs);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hl = lane & 15, lrow0 = warp * 4 + (lane >> 4) * 2;  // rows lrow0, lrow0 + 1
  const int row0 = grp * SCAN_ROWS + lrow0;
  const int slot = slots ? slots[s] : s;
  const int cs = chunk_cu[s], ce = chunk_cu[s + 1];
  const int nseg = seg_cu[s + 1] - seg_cu[s], g = gs - seg_cu[s];
  const int m_seq = cu[s], m_end = cu[s + 1];
  if (slot < 0 || slot >= n_slots || cs < 0 || ce < cs || ce > max_chunks || m_seq < 0 ||
      m_end < m_seq || m_end > M || (m_end - m_seq + CL - 1) / CL != ce - cs ||
      nseg != (ce - cs + SEG - 1) / SEG) {
    if (tid == 0) atomicOr(&g_chunk_bad, 1);
    return;
  }
  // this CTA's segment: chunks [c0, c1), tokens from m_beg
  const int c0 = cs + g * SEG, c1 = min(ce, c0 + SEG);
  const int m_beg = m_seq + g * SEG * CL;
  if (tid == 0) {
    for (int i = 0; i < NSTAGE; ++i) {
      sc_mbar_init(&full[i], 1);
      sc_mbar_init(&empty[i], SCAN_THREADS / 32);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  float* Srow = rnn + (((size_t)slot * H + h) * KD + row0) * KD + 4 * hl;
  float4 st0 = make_float4(0.f, 0.f, 0.f, 0.f), st1 = st0;
  if (g == 0) {
    st0 = *reinterpret_cast<const float4*>(Srow);
    st1 = *reinterpret_cast<const float4*>(Srow + KD);
  }
  // the lane's four reduced sums: row my_row, outputs (my_y) or in-chunk states, t = my_t..+3
  const int my_row = hl < 8 ? row0 : row0 + 1, my_lrow = hl < 8 ? lrow0 : lrow0 + 1;
  const bool my_y = hl & 4;
  const int my_t = (4 * hl) & 15;
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
    const float* RW = R + SHARED_F;
    const float2 a01 = make_float2(st0.x, st0.y), a23 = make_float2(st0.z, st0.w);
    const float2 b01 = make_float2(st1.x, st1.y), b23 = make_float2(st1.z, st1.w);
    // each What / Q load serves both rows of the half-warp
    float p[64];
#pragma unroll
    for (int t = 0; t < CL; ++t) {
      const float4 w = *reinterpret_cast<const float4*>(R + OFF_W + t * KD + 4 * hl);
      const float4 q = *reinterpret_cast<const float4*>(R + OFF_Q + t * KD + 4 * hl);
      p[t] = dot4(w, a01, a23);
      p[CL + t] = dot4(q, a01, a23);
      p[2 * CL + t] = dot4(w, b01, b23);
      p[3 * CL + t] = dot4(q, b01, b23);
    }
    // transpose-reduce over the 16 lanes of the half-warp: 64 -> 32 -> 16 -> 8 -> 4 sums
#pragma unroll
    for (int m = 8, half = 32; m >= 1; m >>= 1, half >>= 1) {
      const bool up = lane & m;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = up ? p[i] : p[i + half];
        const float keep = up ? p[i + half] : p[i];
        p[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
      }
    }
    // lane hl holds sums 4hl..4hl+3 (What s or Q s of row my_row); add PU v / PY v
    const float4 add = *reinterpret_cast<const float4*>(RW + my_lrow * RWS + ((4 * hl) & 31));
    const float4 o = make_float4(p[0] + add.x, p[1] + add.y, p[2] + add.z, p[3] + add.w);
    if (my_y) {
      const int m0 = m_beg + it * CL + my_t;
      const float ov[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (m0 + e >= m_end) break;
        const size_t off = (size_t)(m0 + e) * C + h * KD + my_row;
        if (g == 0) ybuf[off] = f2h(ov[e]);   // final outputs
        else yf32[off] = ov[e];                // partial: k_seg_fix adds the incoming state's part
      }
    }
    const float4 gl = *reinterpret_cast<const float4*>(R + OFF_G + 4 * hl);
    const float4 u0 = *reinterpret_cast<const float4*>(RW + lrow0 * RWS + 2 * CL + 4 * hl);
    const float4 u1 = *reinterpret_cast<const float4*>(RW + (lrow0 + 1) * RWS + 2 * CL + 4 * hl);
    const float2 g01 = make_float2(gl.x, gl.y), g23 = make_float2(gl.z, gl.w);
    float2 n01 = __ffma2_rn(a01, g01, make_float2(u0.x, u0.y));
    float2 n23 = __ffma2_rn(a23, g23, make_float2(u0.z, u0.w));
    float2 m01 = __ffma2_rn(b01, g01, make_float2(u1.x, u1.y));
    float2 m23 = __ffma2_rn(b23, g23, make_float2(u1.z, u1.w));
    const int src0 = lane & 16, src1 = src0 + 8;  // lanes holding the states of row 0 / row 1
#pragma unroll
    for (int j = 0; j < CL; ++j) {
      const float v = (j & 3) == 0 ? o.x : (j & 3) == 1 ? o.y : (j & 3) == 2 ? o.z : o.w;
      const float sa0 = __shfl_sync(0xffffffffu, v, src0 + (j >> 2));
      const float sa1 = __shfl_sync(0xffffffffu, v, src1 + (j >> 2));
      const float4 b = *reinterpret_cast<const float4*>(R + OFF_B + j * KD + 4 * hl);
      const float2 bl = make_float2(b.x, b.y), bh = make_float2(b.z, b.w);
      n01 = __ffma2_rn(make_float2(sa0, sa0), bl, n01);
      n23 = __ffma2_rn(make_float2(sa0, sa0), bh, n23);
      m01 = __ffma2_rn(make_float2(sa1, sa1), bl, m01);
      m23 = __ffma2_rn(make_float2(sa1, sa1), bh, m23);
    }
    st0 = make_float4(n01.x, n01.y, n23.x, n23.y);
    st1 = make_float4(m01.x, m01.y, m23.x, m23.y);
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
  float* dst = nseg == 1 ? Srow : lbuf + (((size_t)gs * H + h) * KD + row0) * KD + 4 * hl;
  *reinterpret_cast<float4*>(dst) = st0;
  *reinterpret_cast<float4*>(dst + KD) = st1;
}

// ---- two-level scan: segment transfers, the cross-segment pass, output correction ----
//
// Chunk map of one state row s (a vector over keys), from the chunk record:
//   s' = A s + u,  A = diag(gL) + Bt^T What   (u: the value terms, independent of s)
// so a segment's true start state S_g (64 rows) reaches chunk c as Phi_c S_g + (the
// zero-start scan), Phi_c = A_{c-1} ... A_{first}, and the chunk's outputs gain
// (Q_c Phi_c) S_g. All fp32.

// 3xTF32 tensor-core products (mma.sync m16n8k8 .tf32, fp32 accumulation): every fp32
// operand x = hi + lo with hi = tf32(x), lo = tf32(x - hi); a product sums
// lo*hi + hi*lo + hi*hi, which keeps about fp32 accuracy.
__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hi) : "f"(x));
  const float r = x - __uint_as_float(hi);
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lo) : "f"(r));
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// d += A B with A (16 x 8) given as fp32 a[4] and B (8 x 8) as fp32 b[2] in the m16n8k8
// fragment layout (g = lane >> 2, q = lane & 3: a0 (g, q), a1 (g+8, q), a2 (g, q+4),
// a3 (g+8, q+4); b0 (k = q, n = g), b1 (k = q+4, n = g); d0/d1 (g, 2q / 2q+1),
// d2/d3 (g+8, 2q / 2q+1)).
__device__ __forceinline__ void mma3_tf32(float (&d)[4], const float (&a)[4], const float (&b)[2]) {
  uint32_t ah[4], al[4], bh[2], bl[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) tf32_split(a[i], ah[i], al[i]);
#pragma unroll
  for (int i = 0; i < 2; ++i) tf32_split(b[i], bh[i], bl[i]);
  mma_tf32(d, al, bh);
  mma_tf32(d, ah, bl);
  mma_tf32(d, ah, bh);
}

constexpr int PH_LD = 72;   // padded row strides: conflict-free fragment loads
constexpr int WQ_LD = 68;

// grid = (max segments, H), block = 256 (8 warps). For every segment of a multi-segment
// sequence: qt[c] = Q_c Phi_c for each of its chunks and phi[seg] = the whole transfer,
// with Phi <- diag(gL) Phi + Bt^T (What Phi) per chunk, all products on the tensor cores
// (3xTF32). The next chunk's record rows travel in registers while one computes.
__device__ __forceinline__ void seg_phi_body(int gs, int h, int H, float* smem,
                                             const float* __restrict__ rec,
                                             const int* __restrict__ chunk_cu,
                                             const int* __restrict__ seg_cu, int S,
                                             float* __restrict__ qt, float* __restrict__ phi) {
  float* Ph = smem;                          // [64][PH_LD]
  float* Am = Ph + KD * PH_LD;               // [32][WQ_LD]: rows 0..15 What, 16..31 Q
  float* Bm = Am + 2 * CL * WQ_LD;           // [16][PH_LD]
  float* X = Bm + CL * PH_LD;                // [16][PH_LD]
  float* gl = X + CL * PH_LD;                // [64]
  const int tid = threadIdx.x;
  if (gs >= seg_cu[S]) return;
  const int s = seq_of(seg_cu, S, gs);
  const int nseg = seg_cu[s + 1] - seg_cu[s];
  if (nseg < 2) return;
  const int g = gs - seg_cu[s];
  const int c0 = chunk_cu[s] + g * SEG, c1 = min(chunk_cu[s + 1], c0 + SEG);
  const int lane = tid & 31, warp = tid >> 5, gq = lane >> 2, q = lane & 3;
  for (int i = tid; i < KD * KD; i += 256) Ph[(i / KD) * PH_LD + i % KD] = (i / KD == i % KD) ? 1.f : 0.f;
  float4 nw, nq, nb;
  float ng = 0.f;
  auto fetch = [&](int c) {
    const float* R = rec + ((size_t)c * H + h) * REC;
    nw = reinterpret_cast<const float4*>(R + OFF_W)[tid];
    nq = reinterpret_cast<const float4*>(R + OFF_Q)[tid];
    nb = reinterpret_cast<const float4*>(R + OFF_B)[tid];
    if (tid < KD) ng = R[OFF_G + tid];
  };
  fetch(c0);
  // step 1 tiles: m-tile (warp >> 2) of [What; Q], n-tiles 2 (warp & 3) and +1
  const int m1 = warp >> 2, n1 = (warp & 3) * 16;
  // step 2 tiles: m-tile (warp >> 1) of the 64 key rows, n-tiles 32 (warp & 1) .. +3
  const int m2 = (warp >> 1) * 16, n2 = (warp & 1) * 32;
  for (int c = c0; c < c1; ++c) {
    {
      const int r = tid >> 4, cc = (tid & 15) * 4;  // record rows are [16][64]
      *reinterpret_cast<float4*>(Am + r * WQ_LD + cc) = nw;
      *reinterpret_cast<float4*>(Am + (CL + r) * WQ_LD + cc) = nq;
      *reinterpret_cast<float4*>(Bm + r * PH_LD + cc) = nb;
      if (tid < KD) gl[tid] = ng;
    }
    __syncthreads();
    if (c + 1 < c1) fetch(c + 1);
    // step 1: [What; Q] (32 x 64) x Phi (64 x 64)
    float d1[2][4] = {};
#pragma unroll
    for (int kb = 0; kb < KD; kb += 8) {
      const float* A = Am + (m1 * 16) * WQ_LD + kb;
      const float a[4] = {A[gq * WQ_LD + q], A[(gq + 8) * WQ_LD + q], A[gq * WQ_LD + q + 4],
                          A[(gq + 8) * WQ_LD + q + 4]};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int nb0 = n1 + nt * 8;
        const float b[2] = {Ph[(kb + q) * PH_LD + nb0 + gq], Ph[(kb + q + 4) * PH_LD + nb0 + gq]};
        mma3_tf32(d1[nt], a, b);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int col = n1 + nt * 8 + 2 * q;
      if (m1 == 0) {  // X = What Phi
        *reinterpret_cast<float2*>(X + gq * PH_LD + col) = make_float2(d1[nt][0], d1[nt][1]);
        *reinterpret_cast<float2*>(X + (gq + 8) * PH_LD + col) = make_float2(d1[nt][2], d1[nt][3]);
      } else {        // Q Phi of this chunk
        float* o = qt + ((size_t)c * H + h) * (CL * KD);
        *reinterpret_cast<float2*>(o + gq * KD + col) = make_float2(d1[nt][0], d1[nt][1]);
        *reinterpret_cast<float2*>(o + (gq + 8) * KD + col) = make_float2(d1[nt][2], d1[nt][3]);
      }
    }
    __syncthreads();
    // step 2: Phi <- diag(gL) Phi + Bt^T X, A[k][t] = Bt[t][k], B[t][j] = X[t][j]
    float d2[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int col = n2 + nt * 8 + 2 * q;
      const float g0 = gl[m2 + gq], g8 = gl[m2 + gq + 8];
      d2[nt][0] = g0 * Ph[(m2 + gq) * PH_LD + col];
      d2[nt][1] = g0 * Ph[(m2 + gq) * PH_LD + col + 1];
      d2[nt][2] = g8 * Ph[(m2 + gq + 8) * PH_LD + col];
      d2[nt][3] = g8 * Ph[(m2 + gq + 8) * PH_LD + col + 1];
    }
#pragma unroll
    for (int kt = 0; kt < CL; kt += 8) {
      const float a[4] = {Bm[(kt + q) * PH_LD + m2 + gq], Bm[(kt + q) * PH_LD + m2 + gq + 8],
                          Bm[(kt + q + 4) * PH_LD + m2 + gq], Bm[(kt + q + 4) * PH_LD + m2 + gq + 8]};
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int nb0 = n2 + nt * 8;
        const float b[2] = {X[(kt + q) * PH_LD + nb0 + gq], X[(kt + q + 4) * PH_LD + nb0 + gq]};
        mma3_tf32(d2[nt], a, b);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int col = n2 + nt * 8 + 2 * q;
      *reinterpret_cast<float2*>(Ph + (m2 + gq) * PH_LD + col) = make_float2(d2[nt][0], d2[nt][1]);
      *reinterpret_cast<float2*>(Ph + (m2 + gq + 8) * PH_LD + col) = make_float2(d2[nt][2], d2[nt][3]);
    }
    __syncthreads();
  }
  float* out = phi + ((size_t)gs * H + h) * (KD * KD);
  for (int i = tid; i < KD * KD / 4; i += 256) {
    const int r = i / (KD / 4), cc = (i % (KD / 4)) * 4;
    reinterpret_cast<float4*>(out)[i] = *reinterpret_cast<const float4*>(Ph + r * PH_LD + cc);
  }
}

static_assert(KD * PH_LD + 2 * CL * WQ_LD + 2 * CL * PH_LD + KD <= NSTAGE * STAGE_F,
              "the transfer-matrix blocks fit the scan's shared memory");

// One launch, two roles, because the transfer matrices need only the chunk records:
// blocks [0, n_phi) are (segment, head) transfer-matrix blocks (seg_phi_body, tensor
// pipe), the rest are (segment, head, row group) scan blocks (chunk_scan_body, a
// latency-bound chain); sharing the SMs, the first hide under the second.
#ifndef SCAN_MINB
#define SCAN_MINB 3
#endif
__global__ void __launch_bounds__(SCAN_THREADS, SCAN_MINB) k_scan_phi(
    const float* __restrict__ rec, const int* __restrict__ cu, const int* __restrict__ chunk_cu,
    const int* __restrict__ seg_cu, const int* __restrict__ slots, float* __restrict__ rnn,
    __half* __restrict__ ybuf, float* __restrict__ yf32, float* __restrict__ lbuf,
    float* __restrict__ qt, float* __restrict__ phi, int S, int H, int C, int M, int max_chunks,
    int n_slots, int n_phi) {
  RWKV_GRID_DEP_ENTRY();
  extern __shared__ __align__(128) float smem[];
  const int bx = blockIdx.x;
  if (bx < n_phi) {
    seg_phi_body(bx / H, bx % H, H, smem, rec, chunk_cu, seg_cu, S, qt, phi);
    return;
  }
  constexpr int G = KD / SCAN_ROWS;
  const int b = bx - n_phi, gs = b / (H * G), rem = b % (H * G);
  chunk_scan_body(gs, rem / G, H, rem % G, smem, rec, cu, chunk_cu, seg_cu, slots, rnn, ybuf,
                  yf32, lbuf, S, C, M, max_chunks, n_slots);
}

// ---- segment scan on the tensor cores (tcgen05, kind::tf32) --------------------------
//
// One CTA per (segment, head), 256 threads; thread (row, half): row = TMEM lane (its
// warp's lane quadrant), half = keys 32 half .. + 31 of that row of a 128 x 64 fp32 state
// block. Rows 0..63 are the head's state rows (the true state for a sequence's first
// segment, zero for the others); rows 64..127 basis rows e_j (later segments only), which
// carry no value terms. Per chunk, the 16 + 16 dot products of every row with What and Q
// are ONE tcgen05.mma chain, M = 128, N = 32, K = 64: the state block is the A operand in
// TMEM (written by its threads with tcgen05.st), [What; Q] the B operand in shared memory;
// every fp32 operand is split into tf32 hi + lo and D = A_lo B_hi + A_hi B_lo + A_hi B_hi
// accumulates in fp32 (about fp32 accuracy). A row's D gives its in-chunk states
// sa = What s + PU v and outputs y = Q s + PY v; the state then advances on the CUDA
// cores, s <- s * gL + U + sum_t sa_t Bt_t. For a basis row j the outputs are column j of
// Q_c Phi_c (qt, for k_seg_fix) and its final state column j of the segment's transfer
// matrix (phi, for k_seg_combine): the transfer matrices come out of the same MMAs. Each
// chunk record (row-independent part and every row's value terms) arrives by one bulk
// copy into a two-stage ring.
namespace {
constexpr int TS_ROWS = 128;
constexpr int TS_THREADS = 256;
constexpr uint32_t TS_TMEM_COLS = 256;  // A hi [0, 64), A lo [64, 128), D [128, 160)
constexpr uint32_t TS_B_BLK = 2 * CL * 128;       // 4 KiB: a 32-wide K-block of [What; Q]
constexpr uint32_t TS_OFF_BHI = 0, TS_OFF_BLO = 2 * TS_B_BLK;
constexpr uint32_t TS_OFF_REC = 4 * TS_B_BLK;
constexpr uint32_t TS_REC_BYTES = REC * 4;
constexpr uint32_t TS_OFF_BAR = TS_OFF_REC + 2 * TS_REC_BYTES;
}  // namespace
constexpr size_t TS_SMEM = 1024 + TS_OFF_BAR + 64;

// byte offset of element (row r, column kk < 32) in a 128-byte swizzled K-major block
__device__ __forceinline__ uint32_t ts_sw(int r, int kk) {
  return (uint32_t)(((r >> 3) << 10) + ((r & 7) << 7) + ((((kk >> 2) ^ (r & 7))) << 4) + ((kk & 3) << 2));
}
__device__ __forceinline__ uint64_t ts_desc(uint32_t saddr_tile) {
  uint64_t d = (uint64_t)((saddr_tile >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;            // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;            // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;            // 128-byte swizzle
  return d;
}
__device__ __forceinline__ void ts_st4(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
__device__ __forceinline__ uint32_t ts_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
// 16 consecutive 32-bit TMEM columns of this thread's lane <- v
__device__ __forceinline__ void ts_tst16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void ts_tld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15},"
      " [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(TS_THREADS, 2) k_seg_scan_tc(
    const float* __restrict__ rec, const int* __restrict__ cu, const int* __restrict__ chunk_cu,
    const int* __restrict__ seg_cu, const int* __restrict__ slots, float* __restrict__ rnn,
    __half* __restrict__ ybuf, float* __restrict__ yf32, float* __restrict__ lbuf,
    float* __restrict__ qt, float* __restrict__ phi, int S, int H, int C, int M, int max_chunks,
    int n_slots) {
  RWKV_GRID_DEP_ENTRY();
  extern __shared__ unsigned char ts_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(ts_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = sm_addr(base);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + TS_OFF_BAR);  // [2] record stages
  uint64_t* mma_bar = full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int gs = blockIdx.x / H, h = blockIdx.x % H;
  if (gs >= seg_cu[S]) return;
  const int s = seq_of(seg_cu, S, gs);
  const int slot = slots ? slots[s] : s;
  const int cs = chunk_cu[s], ce = chunk_cu[s + 1];
  const int nseg = seg_cu[s + 1] - seg_cu[s], g = gs - seg_cu[s];
  const int m_seq = cu[s], m_end = cu[s + 1];
  if (slot < 0 || slot >= n_slots || cs < 0 || ce < cs || ce > max_chunks || m_seq < 0 ||
      m_end < m_seq || m_end > M || (m_end - m_seq + CL - 1) / CL != ce - cs ||
      nseg != (ce - cs + SEG - 1) / SEG) {
    if (tid == 0) atomicOr(&g_chunk_bad, 1);
    return;
  }
  const int c0 = cs + g * SEG, c1 = min(ce, c0 + SEG);
  const int m_beg = m_seq + g * SEG * CL;
  const int row = tid & (TS_ROWS - 1), half = tid >> 7, k0 = 32 * half;
  const bool basis = row >= KD, need_basis = g > 0;  // basis rows matter for later segments
  const int vrow = row & (KD - 1);

  if (tid == 0) {
    sc_mbar_init(&full[0], 1);
    sc_mbar_init(&full[1], 1);
    sc_mbar_init(mma_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     sm_addr(tmem_slot)), "r"(TS_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);

  int issued = 0, waited = 0;  // record copies issued (thread 0) / waited for
  auto issue = [&](int c) {
    const int buf = (c - c0) & 1;
    sc_mbar_expect_tx(&full[buf], TS_REC_BYTES);
    sc_bulk_g2s(base + TS_OFF_REC + buf * TS_REC_BYTES, rec + ((size_t)c * H + h) * REC,
                TS_REC_BYTES, &full[buf]);
    ++issued;
  };
  if (tid == 0) issue(c0);

  // this thread's half row of the state block
  float st[32];
  if (!basis && g == 0) {
    const float4* S0 =
        reinterpret_cast<const float4*>(rnn + (((size_t)slot * H + h) * KD + vrow) * KD + k0);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 v = S0[q];
      st[4 * q] = v.x; st[4 * q + 1] = v.y; st[4 * q + 2] = v.z; st[4 * q + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 32; ++k) st[k] = (basis && need_basis && k0 + k == vrow) ? 1.f : 0.f;
  }

  const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(2 * CL >> 3) << 17) |
                         ((uint32_t)(TS_ROWS >> 4) << 24);   // N = 32: [What; Q]
  const uint32_t idesc2 = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(KD >> 3) << 17) |
                          ((uint32_t)(TS_ROWS >> 4) << 24);  // N = 64: Bt^T
  bool ok = true;
  for (int c = c0; c < c1; ++c) {
    const int it = c - c0, buf = it & 1;
    // the other stage is free (its chunk's readers passed the last barrier): next record
    if (tid == 0 && c + 1 < c1) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(c + 1);
    }
    // A: this half row as tf32 hi / lo into TMEM columns [k0, k0 + 32) and [64 + k0, ..)
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float x = st[16 * p + e];
        hi[e] = ts_tf32(x);
        lo[e] = __float_as_uint(x - __uint_as_float(hi[e]));  // the MMA reads its top 19 bits
      }
      ts_tst16(lane_base + (uint32_t)(k0 + 16 * p), hi);
      ts_tst16(lane_base + (uint32_t)(64 + k0 + 16 * p), lo);
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    // B: [What; Q] of the chunk (32 rows x 64) as tf32 hi / lo, from the record stage
    ok = ok && sc_mbar_wait(&full[buf], (it >> 1) & 1);
    waited += ok ? 1 : 0;
    const float* R = reinterpret_cast<const float*>(base + TS_OFF_REC + buf * TS_REC_BYTES);
    {
      const int n = tid >> 3, kb0 = (tid & 7) * 8;  // 32 rows x 8 pieces of 8
      const float* src = R + (n < CL ? OFF_W + n * KD : OFF_Q + (n - CL) * KD) + kb0;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const float4 v = reinterpret_cast<const float4*>(src)[q];
        const float xs[4] = {v.x, v.y, v.z, v.w};
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          hi[e] = ts_tf32(xs[e]);
          lo[e] = ts_tf32(xs[e] - __uint_as_float(hi[e]));
        }
        const int kk = kb0 + 4 * q;
        const uint32_t o = (kk >> 5) * TS_B_BLK + ts_sw(n, kk & 31);
        ts_st4(sb + TS_OFF_BHI + o, hi[0], hi[1], hi[2], hi[3]);
        ts_st4(sb + TS_OFF_BLO + o, lo[0], lo[1], lo[2], lo[3]);
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      // D = A_lo B_hi + A_hi B_lo + A_hi B_hi over K = 64 (8 steps of K = 8 per pass)
#pragma unroll
      for (int pass = 0; pass < 3; ++pass)
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const uint32_t acol = (pass == 0 ? 64u : 0u) + 32u * kb;
          const uint64_t bd = ts_desc(sb + (pass == 1 ? TS_OFF_BLO : TS_OFF_BHI) + kb * TS_B_BLK);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint32_t accum = (pass | kb | ks) ? 1u : 0u;
            asm volatile(
                "{\n\t.reg .pred p;\n\t"
                "setp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem + 128u),
                "r"(tmem + acol + 8u * ks), "l"(bd + (uint64_t)(2 * ks)), "r"(idesc), "r"(accum));
          }
        }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       sm_addr(mma_bar))
                   : "memory");
    }
    ok = __syncthreads_and(sc_mbar_wait(mma_bar, 0)) != 0;
    if (!ok) break;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // D row: columns 0..15 What s, 16..31 Q s
    float sa[CL], dq[CL];
    ts_tld16(lane_base + 128u, sa);
    ts_tld16(lane_base + 128u + CL, dq);
    const float* RW = R + OFF_RW + vrow * RWS;  // this state row's value terms
    if (!basis) {
#pragma unroll
      for (int q = 0; q < CL / 4; ++q) {
        const float4 a = reinterpret_cast<const float4*>(RW)[q];
        sa[4 * q] += a.x; sa[4 * q + 1] += a.y; sa[4 * q + 2] += a.z; sa[4 * q + 3] += a.w;
      }
    }
    // the second product, sum_t sa_t Bt_t (M = 128, N = 64, K = 16): sa as tf32 hi / lo into
    // TMEM columns [0, 16) / [64, 80) (the first half of each row), Bt^T into the B tiles
    if (half == 0) {
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        hi[e] = ts_tf32(sa[e]);
        lo[e] = __float_as_uint(sa[e] - __uint_as_float(hi[e]));
      }
      ts_tst16(lane_base, hi);
      ts_tst16(lane_base + 64u, lo);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    {
      const int n = tid >> 2, t0 = (tid & 3) * 4;  // 64 rows n (keys) x 4 groups of 4 t
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float x = R[OFF_B + (t0 + e) * KD + n];
        hi[e] = ts_tf32(x);
        lo[e] = __float_as_uint(x - __uint_as_float(hi[e]));
      }
      const uint32_t o = ts_sw(n, t0);
      ts_st4(sb + TS_OFF_BHI + o, hi[0], hi[1], hi[2], hi[3]);
      ts_st4(sb + TS_OFF_BLO + o, lo[0], lo[1], lo[2], lo[3]);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
      for (int pass = 0; pass < 3; ++pass) {
        const uint32_t acol = pass == 0 ? 64u : 0u;
        const uint64_t bd = ts_desc(sb + (pass == 1 ? TS_OFF_BLO : TS_OFF_BHI));
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const uint32_t accum = (pass | ks) ? 1u : 0u;
          asm volatile(
              "{\n\t.reg .pred p;\n\t"
              "setp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem + 160u),
              "r"(tmem + acol + 8u * ks), "l"(bd + (uint64_t)(2 * ks)), "r"(idesc2), "r"(accum));
        }
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       sm_addr(mma_bar))
                   : "memory");
    }
    // outputs while the second product runs (the first half of each row writes them)
    const int mc = m_beg + it * CL;  // first token of the chunk
    if (!basis) {
      if (half == 0) {
        const int nt = min(CL, m_end - mc);
        float y[CL];
#pragma unroll
        for (int q = 0; q < CL / 4; ++q) {
          const float4 b = reinterpret_cast<const float4*>(RW + CL)[q];
          y[4 * q] = dq[4 * q] + b.x; y[4 * q + 1] = dq[4 * q + 1] + b.y;
          y[4 * q + 2] = dq[4 * q + 2] + b.z; y[4 * q + 3] = dq[4 * q + 3] + b.w;
        }
        if (g == 0) {
          __half* yp = ybuf + (size_t)mc * C + h * KD + vrow;  // final outputs
#pragma unroll
          for (int t = 0; t < CL; ++t) {
            if (t < nt) *yp = f2h(y[t]);
            yp += C;
          }
        } else {
          float* yp = yf32 + (size_t)mc * C + h * KD + vrow;  // partial: k_seg_fix adds
#pragma unroll                                                // the incoming state's part
          for (int t = 0; t < CL; ++t) {
            if (t < nt) *yp = y[t];
            yp += C;
          }
        }
      }
    } else if (need_basis && half == 0) {
      float* q = qt + ((size_t)c * H + h) * (CL * KD) + vrow;
#pragma unroll
      for (int t = 0; t < CL; ++t) q[t * KD] = dq[t];
    }
    // s <- s * gL + U + sum_t sa_t Bt_t over this thread's keys
    ok = __syncthreads_and(sc_mbar_wait(mma_bar, 1)) != 0;
    if (!ok) break;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    {
      float d2[32];
      ts_tld16(lane_base + 160u + k0, *reinterpret_cast<float(*)[16]>(d2));
      ts_tld16(lane_base + 160u + k0 + 16, *reinterpret_cast<float(*)[16]>(d2 + 16));
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      const float4* gl4 = reinterpret_cast<const float4*>(R + OFF_G + k0);
      const float4* U4 = reinterpret_cast<const float4*>(RW + 2 * CL + k0);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 gq = gl4[q];
        const float4 u = basis ? make_float4(0.f, 0.f, 0.f, 0.f) : U4[q];
        st[4 * q] = fmaf(st[4 * q], gq.x, u.x) + d2[4 * q];
        st[4 * q + 1] = fmaf(st[4 * q + 1], gq.y, u.y) + d2[4 * q + 1];
        st[4 * q + 2] = fmaf(st[4 * q + 2], gq.z, u.z) + d2[4 * q + 2];
        st[4 * q + 3] = fmaf(st[4 * q + 3], gq.w, u.w) + d2[4 * q + 3];
      }
    }
    __syncthreads();  // the stage, the operands and the accumulator are free again
  }
  if (ok) {
    if (!basis) {
      float* dst = (nseg == 1 ? rnn + (((size_t)slot * H + h) * KD + vrow) * KD
                              : lbuf + (((size_t)gs * H + h) * KD + vrow) * KD) + k0;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        reinterpret_cast<float4*>(dst)[q] = make_float4(st[4 * q], st[4 * q + 1], st[4 * q + 2], st[4 * q + 3]);
    } else if (need_basis) {  // column vrow of the segment's transfer matrix
      float* o = phi + ((size_t)gs * H + h) * (KD * KD) + (size_t)k0 * KD + vrow;
#pragma unroll
      for (int k = 0; k < 32; ++k) o[k * KD] = st[k];
    }
  } else if (tid == 0) {
    // leave no bulk copy in flight into this CTA's shared memory
    for (int i = waited; i < issued; ++i) sc_mbar_wait(&full[i & 1], (i >> 1) & 1);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TS_TMEM_COLS));
}

// grid = (S, H, 4 row quarters), block = 256. Walks a multi-segment sequence's segments
// in order: the true start of segment g + 1 is phi[g] applied to the true start of g
// plus g's zero-start end state (segment 0's end state, scanned from the true state,
// is already the true start of segment 1). Start states go to sst for k_seg_fix; the final state
// to rnn. Thread: key k = tid & 63, rows 4 (tid >> 6) .. +3 of the quarter. The product is
// bound by shared-memory wavefronts, so both operands are read 16 bytes at a time: a row
// of Phi four columns per load, and the quarter's state stored transposed so that the four
// rows a thread updates come in one broadcast load. Each sum still runs in j order.
constexpr int CMB_PLD = KD + 4;  // Phi row stride: 8 lanes' 16-byte loads on distinct banks
constexpr int CMB_SLD = 16 + 4;  // transposed state row stride (16 rows + pad), same reason
__global__ void __launch_bounds__(256) k_seg_combine(const int* __restrict__ seg_cu,
                                                     const int* __restrict__ slots,
                                                     const float* __restrict__ lbuf,
                                                     const float* __restrict__ phi,
                                                     float* __restrict__ sst,
                                                     float* __restrict__ rnn) {
  RWKV_GRID_DEP_ENTRY();
  __shared__ __align__(16) float Ps[KD * CMB_PLD];  // Phi[k][j] at k * CMB_PLD + j
  __shared__ __align__(16) float St[KD * CMB_SLD];  // state row v, column j at j * CMB_SLD + v
  const int s = blockIdx.x, h = blockIdx.y, H = gridDim.y, q = blockIdx.z, tid = threadIdx.x;
  const int seg0 = seg_cu[s], nseg = seg_cu[s + 1] - seg0;
  if (nseg < 2) return;
  const int slot = slots ? slots[s] : s;
  const int k = tid & 63, v0 = (tid >> 6) * 4;  // rows v0..v0+3 of the quarter
  const size_t rbase = (size_t)(q * 16) * KD;   // first row of the quarter
  auto seg_off = [&](int g) { return ((size_t)(seg0 + g) * H + h) * KD * KD; };
  float st[4], pl[4], pp[16];  // state; prefetched L_g and Phi_g of the next step
  const size_t o0 = seg_off(0);
#pragma unroll
  for (int e = 0; e < 4; ++e) st[e] = lbuf[o0 + rbase + (v0 + e) * KD + k];
  auto fetch = [&](int g) {
    const size_t so = seg_off(g);
#pragma unroll
    for (int e = 0; e < 4; ++e) pl[e] = lbuf[so + rbase + (v0 + e) * KD + k];
#pragma unroll
    for (int i = 0; i < 16; ++i) pp[i] = phi[so + tid + 256 * i];
  };
  fetch(1);
  for (int g = 1; g < nseg; ++g) {
    const size_t so = seg_off(g);
#pragma unroll
    for (int e = 0; e < 4; ++e) sst[so + rbase + (v0 + e) * KD + k] = st[e];
    *reinterpret_cast<float4*>(St + k * CMB_SLD + v0) = make_float4(st[0], st[1], st[2], st[3]);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int idx = tid + 256 * i;
      Ps[(idx / KD) * CMB_PLD + idx % KD] = pp[i];
    }
    float acc[4] = {pl[0], pl[1], pl[2], pl[3]};
    __syncthreads();
    if (g + 1 < nseg) fetch(g + 1);
    // start of segment g + 1 = Phi_g (start of g) + (g's zero-start end state)
    const float4* P4 = reinterpret_cast<const float4*>(Ps + k * CMB_PLD);
#pragma unroll 4
    for (int j4 = 0; j4 < KD / 4; ++j4) {
      const float4 p4 = P4[j4];
      const float pj[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const float4 s4 = *reinterpret_cast<const float4*>(St + (4 * j4 + jj) * CMB_SLD + v0);
        acc[0] += pj[jj] * s4.x;
        acc[1] += pj[jj] * s4.y;
        acc[2] += pj[jj] * s4.z;
        acc[3] += pj[jj] * s4.w;
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) st[e] = acc[e];
    __syncthreads();
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) rnn[(((size_t)slot * H + h) * KD) * KD + rbase + (v0 + e) * KD + k] = st[e];
}

// grid = (max segments, H), block = 256 (8 warps). Segments g >= 1 of multi-segment
// sequences: for each chunk, y = yf32 + (Q Phi) S_g^T on the tensor cores (3xTF32),
// rounded to fp16 once (like the reference's y store). Warp w owns state rows 8w..8w+7;
// S_g is loaded once per segment, the next chunk's Q Phi and fp32 partial outputs are
// prefetched into registers.
__global__ void __launch_bounds__(256) k_seg_fix(const int* __restrict__ cu,
                                                 const int* __restrict__ chunk_cu,
                                                 const int* __restrict__ seg_cu, int S,
                                                 const float* __restrict__ qt,
                                                 const float* __restrict__ sst,
                                                 const float* __restrict__ yf32,
                                                 __half* __restrict__ ybuf, int C) {
  RWKV_GRID_DEP_ENTRY();
  __shared__ __align__(16) float Ss[KD * WQ_LD];
  __shared__ __align__(16) float Qs[CL * WQ_LD];
  // blockIdx.x = segment * (SEG / FIX_CHUNKS) + part: each CTA corrects FIX_CHUNKS
  // chunks of one segment, so the chunks of a segment are corrected in parallel
  const int gs = blockIdx.x / (SEG / FIX_CHUNKS), part = blockIdx.x % (SEG / FIX_CHUNKS);
  const int h = blockIdx.y, H = gridDim.y, tid = threadIdx.x;
  if (gs >= seg_cu[S]) return;
  const int s = seq_of(seg_cu, S, gs);
  const int nseg = seg_cu[s + 1] - seg_cu[s], g = gs - seg_cu[s];
  if (nseg < 2 || g == 0) return;
  const int cseg = chunk_cu[s] + g * SEG;
  const int c0 = cseg + part * FIX_CHUNKS;
  const int c1 = min(min(chunk_cu[s + 1], cseg + SEG), c0 + FIX_CHUNKS);
  if (c0 >= c1) return;
  const size_t so = ((size_t)gs * H + h) * KD * KD;
  for (int i = tid; i < KD * KD / 4; i += 256) {
    const int r = i / (KD / 4), cc = (i % (KD / 4)) * 4;
    *reinterpret_cast<float4*>(Ss + r * WQ_LD + cc) = reinterpret_cast<const float4*>(sst + so)[i];
  }
  const int lane = tid & 31, warp = tid >> 5, gq = lane >> 2, q = lane & 3;
  const int m_end = cu[s + 1];
  const int nb0 = warp * 8, v = nb0 + 2 * q;
  // a chunk's fp32 partial outputs (rows gq and gq + 8 of the chunk, columns v, v + 1)
  auto load_y = [&](int c, float2 (&yv)[2]) {
    const int m0 = cu[s] + (c - chunk_cu[s]) * CL;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int m = m0 + gq + 8 * half;
      yv[half] = m < m_end ? *reinterpret_cast<const float2*>(yf32 + (size_t)m * C + h * KD + v)
                           : make_float2(0.f, 0.f);
    }
  };
  // Q Phi and the partial outputs of the next chunk are fetched one chunk ahead
  float4 nq = reinterpret_cast<const float4*>(qt + ((size_t)c0 * H + h) * (CL * KD))[tid];
  float2 yv[2], ny[2];
  load_y(c0, ny);
  for (int c = c0; c < c1; ++c) {
    *reinterpret_cast<float4*>(Qs + (tid >> 4) * WQ_LD + (tid & 15) * 4) = nq;
    yv[0] = ny[0];
    yv[1] = ny[1];
    __syncthreads();
    if (c + 1 < c1) {
      nq = reinterpret_cast<const float4*>(qt + ((size_t)(c + 1) * H + h) * (CL * KD))[tid];
      load_y(c + 1, ny);
    }
    const int m0 = cu[s] + (c - chunk_cu[s]) * CL;
    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kb = 0; kb < KD; kb += 8) {
      const float a[4] = {Qs[gq * WQ_LD + kb + q], Qs[(gq + 8) * WQ_LD + kb + q],
                          Qs[gq * WQ_LD + kb + q + 4], Qs[(gq + 8) * WQ_LD + kb + q + 4]};
      const float b[2] = {Ss[(nb0 + gq) * WQ_LD + kb + q], Ss[(nb0 + gq) * WQ_LD + kb + q + 4]};
      mma3_tf32(d, a, b);
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int m = m0 + gq + 8 * half;
      if (m < m_end)
        *reinterpret_cast<__half2*>(ybuf + (size_t)m * C + h * KD + v) =
            __floats2half2_rn(yv[half].x + d[2 * half], yv[half].y + d[2 * half + 1]);
    }
    __syncthreads();
  }
}

namespace {
// V consecutive fp16 channels (V = 2: 4-byte, V = 8: 16-byte access) as floats.
template <int V>
__device__ __forceinline__ void ld_ch(const __half* p, float (&v)[V]) {
  if constexpr (V == 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(p));
    v[0] = f.x;
    v[1] = f.y;
  }
}
// Caller vectors (r_k, ln_x weights): 4-byte loads whatever V.
template <int V>
__device__ __forceinline__ void ld_ch_user(const __half* p, float (&v)[V]) {
#pragma unroll
  for (int i = 0; i < V / 2; ++i) {
    const float2 f = __half22float2(reinterpret_cast<const __half2*>(p)[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
}  // namespace

// Per-head GroupNorm + bonus + g gate on precomputed y. grid = M rows, block = C / V
// threads, V channels per thread: V = 2 (one warp per head) or, for large batches, V = 8
// (8 lanes per head, 16-byte accesses); the head sums replay warp_sum's tree
// (warp_sum_p), so both round identically.
template <int SEM, int V>
__global__ void k_wkv_epilogue(const __half* __restrict__ ybuf, const __half* __restrict__ rbuf,
                               const __half* __restrict__ gbuf, size_t plane,
                               const __half* __restrict__ r_k, const __half* __restrict__ lnx_w,
                               const __half* __restrict__ lnx_b, __half* __restrict__ yg, int C) {
  RWKV_GRID_DEP_ENTRY();
  constexpr int P = V / 2;
  const int m = blockIdx.x, c = threadIdx.x * V;
  const size_t o = (size_t)m * C + c;
  float y[V], rr[V], kk[V], vv[V], gg[V], rk[V], lw[V], lb[V], p[P];
  ld_ch<V>(ybuf + o, y);
#pragma unroll
  for (int q = 0; q < P; ++q) p[q] = y[2 * q] + y[2 * q + 1];
  const float mean = warp_sum_p<P>(p) * (1.0f / RWKV_HD);
  float d[V];
#pragma unroll
  for (int e = 0; e < V; ++e) d[e] = y[e] - mean;
#pragma unroll
  for (int q = 0; q < P; ++q) p[q] = d[2 * q] * d[2 * q] + d[2 * q + 1] * d[2 * q + 1];
  const float var = warp_sum_p<P>(p) * (1.0f / RWKV_HD);
  const float rstd = 1.0f / sqrtf(var + 64e-5f);
  ld_ch<V>(rbuf + o, rr);
  ld_ch<V>(gbuf + plane + o, kk);
  ld_ch<V>(gbuf + 2 * plane + o, vv);
  ld_ch<V>(gbuf + 5 * plane + o, gg);
  ld_ch_user<V>(r_k + c, rk);
  ld_ch_user<V>(lnx_w + c, lw);
  ld_ch_user<V>(lnx_b + c, lb);
  float out[V];
  if (SEM == SEM_DECODE) {
#pragma unroll
    for (int q = 0; q < P; ++q) {
      p[q] = rr[2 * q] * kk[2 * q] * rk[2 * q];
      p[q] += rr[2 * q + 1] * kk[2 * q + 1] * rk[2 * q + 1];
    }
    const float rkrk = warp_sum_p<P>(p);
#pragma unroll
    for (int e = 0; e < V; ++e) out[e] = r16(d[e] * rstd * lw[e] + lb[e] + rkrk * vv[e]);
  } else {
#pragma unroll
    for (int q = 0; q < P; ++q)
      p[q] = r16(r16(rr[2 * q] * kk[2 * q]) * rk[2 * q]) +
             r16(r16(rr[2 * q + 1] * kk[2 * q + 1]) * rk[2 * q + 1]);
    const float rkrk = r16(warp_sum_p<P>(p));
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const float f = r16(d[e] * rstd * lw[e] + lb[e]);
      out[e] = r16(f + r16(rkrk * vv[e]));
    }
  }
  if constexpr (V == 8) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      h[i] = __floats2half2_rn(out[2 * i] * gg[2 * i], out[2 * i + 1] * gg[2 * i + 1]);
    *reinterpret_cast<uint4*>(yg + o) = u;
  } else {
    *reinterpret_cast<__half2*>(yg + o) = __floats2half2_rn(out[0] * gg[0], out[1] * gg[1]);
  }
}

// Scratch of the chunked recurrence (floats, in this order): chunk records [chunks][H][REC],
// Q Phi per chunk [chunks][H][16 x 64], per segment the zero-start end state, the
// transfer Phi and the true start state [segments][H][64 x 64] each, fp32 outputs
// [M][C], then the segment table (S + 1 ints). chunks <= M/16 + S, segments <= M/(16 SEG) + S.
struct ChunkScratch {
  float *rec, *qt, *lbuf, *phi, *sst, *yf32;
  int* seg_cu;
};
namespace {
size_t pad64(size_t n) { return (n + 63) & ~size_t(63); }
ChunkScratch chunk_scratch(float* base, int M, int S, int H, size_t* total_floats) {
  const size_t maxc = (size_t)M / CL + S, maxs = (size_t)M / (CL * SEG) + S;
  ChunkScratch c;
  size_t o = 0;
  c.rec = base + o;  o += pad64(maxc * H * REC);
  c.qt = base + o;   o += pad64(maxc * H * CL * KD);
  c.lbuf = base + o; o += pad64(maxs * H * KD * KD);
  c.phi = base + o;  o += pad64(maxs * H * KD * KD);
  c.sst = base + o;  o += pad64(maxs * H * KD * KD);
  c.yf32 = base + o; o += pad64((size_t)M * H * KD);
  c.seg_cu = reinterpret_cast<int*>(base + o); o += pad64((size_t)S + 1);
  if (total_floats) *total_floats = o;
  return c;
}
}  // namespace

size_t wkv_chunk_record_bytes(int M, int S, int H) {
  size_t n = 0;
  chunk_scratch(nullptr, M, S, H, &n);
  return n * sizeof(float);
}

// Chunked recurrence only: y (fp16) for every row, state updated in place.
// r..b, y: [M, C] rows (C = H * 64); rnn: [slots, H, 64, 64].
// chunk_cu[s] / seg_cu[s] = chunks / segments before sequence s; they depend on the
// sequence table only, so a forward computes them once for all layers. `rec` is the
// chunk scratch (wkv_chunk_record_bytes(M, S, H) bytes).
int launch_chunk_table(const int* cu, int* chunk_cu, float* rec, int M, int S, int H,
                       cudaStream_t st) {
  const ChunkScratch cs = chunk_scratch(rec, M, S, H, nullptr);
  return rwkv_launch("chunk_table", k_chunk_table, dim3(1), dim3(1024), 0, st, cu, chunk_cu,
                     cs.seg_cu, S);
}

// Chunk transforms + two-level scan of one layer; the tables must already be built.
int launch_wkv_chunked(const __half* r, const __half* w, const __half* k, const __half* v,
                       const __half* a, const __half* b, float* rnn, const int* cu,
                       const int* slots, __half* ybuf, float* rec, int* chunk_cu, int M, int S,
                       int H, int n_slots, cudaStream_t st) {
  const int C = H * KD;
  const ChunkScratch cs = chunk_scratch(rec, M, S, H, nullptr);
  const int maxc = M / CL + S, maxs = M / (CL * SEG) + S;
  int rc;
  if ((rc = rwkv_launch("chunk_prep", k_chunk_prep, dim3(maxc, H), dim3(256), 0, st, r, w, k,
                        v, a, b, cu, chunk_cu, S, C, M, cs.rec)))
    return rc;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_scan_phi, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)SCAN_SMEM);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k_seg_scan_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)TS_SMEM);
    if (e != cudaSuccess) {
      rwkv_set_error("chunk_scan: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return RWKV_ERR_CUDA;
    }
    attr_done[dev] = true;
  }
  // plain launch: thousands of early-placed segment CTAs would crowd the SMs prep runs on
  rwkv_chain_begin();
  // The tensor-core scan's chunk step is a longer dependent chain (two MMA round trips per
  // chunk) than the CUDA-core scan's, and wins once there are enough (segment, head) units
  // to keep two per SM busy (measured on 0.4B: single sequences of T <= 256 favour the
  // CUDA-core scan, T >= 512 and long varlen batches the tensor-core scan).
  // RWKV_B200_SCAN_TC=0 / 1 forces either.
  static const int scan_tc_env = [] {
    const char* e = std::getenv("RWKV_B200_SCAN_TC");
    return e ? (e[0] == '0' ? 0 : 1) : -1;
  }();
  const bool scan_tc = scan_tc_env >= 0 ? scan_tc_env == 1 : maxs * H >= 64;
  if (scan_tc) {
    if ((rc = rwkv_launch("seg_scan_tc", k_seg_scan_tc, dim3(maxs * H), dim3(TS_THREADS), TS_SMEM,
                          st, cs.rec, cu, chunk_cu, cs.seg_cu, slots, rnn, ybuf, cs.yf32,
                          cs.lbuf, cs.qt, cs.phi, S, H, C, M, maxc, n_slots)))
      return rc;
  } else {
    const int n_phi = maxs * H;
    if ((rc = rwkv_launch("scan_phi", k_scan_phi, dim3(n_phi + maxs * H * (KD / SCAN_ROWS)),
                          dim3(SCAN_THREADS), SCAN_SMEM, st, cs.rec, cu, chunk_cu, cs.seg_cu,
                          slots, rnn, ybuf, cs.yf32, cs.lbuf, cs.qt, cs.phi, S, H, C, M, maxc,
                          n_slots, n_phi)))
      return rc;
  }
  if ((rc = rwkv_launch("seg_combine", k_seg_combine, dim3(S, H, 4), dim3(256), 0, st, cs.seg_cu,
                        slots, cs.lbuf, cs.phi, cs.sst, rnn)))
    return rc;
  return rwkv_launch("seg_fix", k_seg_fix, dim3(maxs * (SEG / FIX_CHUNKS), H), dim3(256), 0, st,
                     cu, chunk_cu,
                     cs.seg_cu, S, cs.qt, cs.sst, cs.yf32, ybuf, C);
}

int launch_wkv_epilogue(int sem, const __half* ybuf, const __half* rbuf, const __half* gbuf,
                        size_t plane, const __half* r_k, const __half* lnx_w,
                        const __half* lnx_b, __half* yg, int M, int C, cudaStream_t st) {
  // 8 channels per thread on large batches (C / 8 whole warps)
  const bool wide = rwkv_rows_wide(M, C);
#define EPI_GO(S, V)                                                                           \
  return rwkv_launch("wkv_epilogue", k_wkv_epilogue<S, V>, dim3(M), dim3(C / V), 0, st, ybuf, \
                     rbuf, gbuf, plane, r_k, lnx_w, lnx_b, yg, C)
  if (wide) {
    if (sem == SEM_DECODE) EPI_GO(SEM_DECODE, 8);
    EPI_GO(SEM_PREFILL, 8);
  }
  if (sem == SEM_DECODE) EPI_GO(SEM_DECODE, 2);
  EPI_GO(SEM_PREFILL, 2);
#undef EPI_GO
}

__global__ void k_uniform_cu(int* cu, int S, int T) {
  RWKV_GRID_DEP_ENTRY();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i <= S) cu[i] = i * T;
}

// Self-test of the chunk scan's bounded record wait (sc_mbar_wait) on an mbarrier
// that nothing arrives on: it must give up after SCAN_WAIT_NS, set bit 2 of the
// device error word and return.
namespace {
__global__ void k_wait_selftest_scan(int* out) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    sc_mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    out[0] = sc_mbar_wait(&bar, 0) ? 0 : 1;
  }
}
}  // namespace
int wait_selftest_scan(int* out, cudaStream_t st) {
  return rwkv_launch("wait_selftest_scan", k_wait_selftest_scan, dim3(1), dim3(32), 0, st, out);
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
  // token counts are int inside the kernels: refuse what does not fit
  if ((size_t)n_seq * (size_t)T > (size_t)INT_MAX) return 0;
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
  if ((size_t)n_seq * T * H * KD > ((size_t)1 << 31)) {
    rwkv_set_error("rwkv7_dplr_chunked: problem too large (%d x %d x %d)", n_seq, T, H);
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
  cudaStream_t st = (cudaStream_t)stream;
  int* cu = static_cast<int*>(workspace);
  int* chunk_cu = cu + n_seq + 1;
  float* rec = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                        (((size_t)(n_seq + 1) * 2 * sizeof(int) + 255) & ~size_t(255)));
  int rc = rwkv_launch("uniform_cu", k_uniform_cu, dim3((n_seq + 256) / 256), dim3(256), 0, st, cu,
                       n_seq, T);
  if (rc) return rc;
  if ((rc = launch_chunk_table(cu, chunk_cu, rec, n_seq * T, n_seq, H, st))) return rc;
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
// first call (make that first call before any stream capture). That cached
// address belongs to the device's current context: after cudaDeviceReset in
// the host process it is stale, so do not call this entry point again after a
// device reset in the same process.
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
  if ((size_t)n_seq * T * H * KD > ((size_t)1 << 31)) {
    rwkv_set_error("rwkv7_dplr_chunked_noalloc: problem too large (%d x %d x %d)", n_seq, T, H);
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
