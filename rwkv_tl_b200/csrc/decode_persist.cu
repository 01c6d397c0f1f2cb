// Small-batch decode (one token for each of B <= 4 sequences; layouts for 1, 2 and 4)
// as ONE persistent kernel per step: one CTA per SM, launched cooperatively so that
// every CTA is resident, with a grid barrier between the three phases of each layer
// and before the head.
//
// Cross-CTA sums (the W_o and FFN-value partials) are fixed-point integer atomics
// (fx_add), so a step's results do not depend on the order the CTAs finish in: the
// kernel is bit-reproducible from run to run.
//
// Reference: RWKV7Base.decode and its per-token kernels (demo/_rwkv7_base.py:74-87,
// 153-206, 276-292; src/rwkv_tl/kernels/{lerp,gates,dplr}.py) with the decode rounding
// points -- the same arithmetic, in the same order, as the three-kernel path in
// decode_gemv.cu, except that dot products are summed by tensor-core tiles.
//
// At B = 1 a step streams 0.78 GB of weights through 73 dependent stages. With one
// kernel per stage the launch chain alone costs ~3 us per stage; here a stage boundary
// is a grid barrier (one release-add per CTA and an acquire spin), and every CTA's
// weight slice for the NEXT phase is already in flight into shared memory -- issued by
// one thread to the TMA unit (bulk rows, 2-D / 3-D tensor-map boxes with 128- or
// 64-byte swizzle; no multicast), completing on an mbarrier -- while the current phase
// computes and waits. HBM traffic runs behind the barriers; only activation hand-offs
// (a few KB, L2 resident) sit on the critical path.
//
// The GEMVs run on the tensor cores (mma.sync m16n8k16, fp16 operands, fp32
// accumulation: products are exact, as in an fp32 FMA of fp16 values): with B <= 4
// the fp16 -> fp32 conversions of a CUDA-core dot product, not HBM, would bound them.
// Weight tiles are read with ldmatrix from the swizzled staging layout; the B operand
// is the activation vector (columns past B are zero).
//
//   A(l)  task CTAs x = x1 + fp16(acc2[l-1]) (or the embedding row), LN1, six token-shift
//                   mixes; GEMV over the task's <= 24 rows, all of one mix (r | k | v |
//                   LoRA v | w | a | g rows of [W_rkv ; W_lora_dn])
//   B(l)  GPH CTAs per head  LoRA-up + gates + L2 norm + wkv7 step + GroupNorm/bonus/g,
//                   computed redundantly by the head's CTAs (CTA 0 of the group writes
//                   the state); each then projects its own rows of W_o[:, head]:
//                   acc1[l] += W_o[rows, head] @ yg
//   C(l)  all CTAs  x1 = x + fp16(acc1[l]), LN2, mix, 24..32 FFN key rows -> relu^2 ->
//                   acc2[l] += W_fv[:, rows] @ h
//   head  all CTAs  x1 + fp16(acc2[L-1]), ln_out, logits GEMV (first rows staged, rest
//                   streamed)
// Shared memory (C = 1024, B = 1: 215 KB): A rows | A vectors | B slice, then the FFN
// value slice | B vectors | FFN key rows | C vectors | C activations. The phase-A mixes
// live in the key-row buffer (filled only from phase B on) and the phase-B scratch in
// the A-row buffer (refilled only from phase C on).
//
// Activations written inside the kernel are read with ld.global.cg (L2), never through
// the non-coherent or L1 paths. Every wait is bounded (200 ms): on expiry the kernel
// raises the device error flag and an abort word, every CTA drains its bulk copies and
// returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "decode_common.cuh"

namespace {

using namespace dec;

constexpr int PMAXB = 4;
constexpr int PMAXL = 24;
constexpr int MAXG = 160;  // CTAs (SMs) at most
constexpr int RA = 24;     // phase-A rows per task (multiple of 8)
constexpr int FROWS = 32;  // FFN hidden rows per CTA at most (groups of 8)
constexpr int NREP = 2;    // replicas of the FFN accumulator (CTA c adds into c % NREP; measured: 2 beats 1 and 4)
constexpr uint64_t WAIT_NS = 200000000ull;

struct GridBar {
  unsigned count, abort, pad[2];
};

__device__ int g_persist_timeout = 0;
// Phase timestamps for latency studies (build with -DPERSIST_STAMPS=1): thread 0 of
// every CTA records %globaltimer at fixed points; rwkv7_decode_persist_stamps copies
// them out.
#ifndef PERSIST_STAMPS
#define PERSIST_STAMPS 0
#endif
#if PERSIST_STAMPS
__device__ unsigned long long g_stamp[160 * 256];
#define STAMP(k) do { if (threadIdx.x == 0) { uint64_t t_; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_)); g_stamp[blockIdx.x * 256 + (k)] = t_; } } while (0)
#else
#define STAMP(k) do {} while (0)
#endif

// Phase-A task: rows [row0, row0 + nrows) of W_rkv (src 0) or W_lora_dn (src 1), all
// multiplied by mix vector `mix`.
struct ATask {
  int src, row0, nrows, mix;
};

struct LayerMaps {
  CUtensorMap w_rkv;    // 3-D (64, 3C, C/64) box (64, RA, C/64), 128B swizzle
  CUtensorMap lora_dn;  // 3-D (64, 288, C/64) box (64, RA, C/64), 128B swizzle
  CUtensorMap w_fk;     // 3-D (64, 4C, C/64) box (64, FROWS, C/64), 128B swizzle
  CUtensorMap lora_up;  // 2-D [288, C] box [144, 64], 128B swizzle
  CUtensorMap w_o;      // 2-D [C, C] box [rows_b, 64], 128B swizzle
  CUtensorMap w_fv;     // 2-D [C, 4C] box [256, 32], 64B swizzle
};

struct PParams {
  int B, C, H, L, V, n_slots;
  int n_atask;        // phase-A tasks (CTAs past them idle in phase A)
  int gph, rows_b;    // CTAs per head in phase B, W_o rows per CTA
  int per_v;          // head rows per CTA
  int slot_base;      // slot of sequence b when `slots` is null: slot_base + b
  const int64_t* tokens;
  const int* slots;
  const __half *emb, *head, *lnout_w, *lnout_b;
  __half* logits;
  __half *xln1, *xln2, *rkv, *ranks, *vfirst;
  long long* acc;  // per layer, fixed point (fx_add): acc1 [B][C], then acc2 [NREP][B][C]
  GridBar* bar;
  float* rnn;
  __half *tmix_x, *cmix_x;
  CUtensorMap head_map;  // 3-D (64, V, C/64) box (64, 32, C/64), 128B swizzle
  ATask atask[MAXG];
  DecLayer layers[PMAXL];
  LayerMaps maps[PMAXL];
};

struct SmemLayout {
  size_t a, ac, bv, bc, k, cc, xc, xr, total;
};

__host__ __device__ inline size_t al1k(size_t v) { return (v + 1023) & ~size_t(1023); }
__host__ __device__ inline int mld_of(int C) { return C + 8; }  // padded activation rows

// The sequences' token-shift rows (tmix x for phase A, cmix x for phase C) are staged
// in shared memory with the other vectors for NB <= 2; the four-sequence layout reads
// them from L2 (prefetched one phase ahead) to fit in 227 KB.
__host__ __device__ constexpr int staged_x_rows(int NB) { return NB <= 2 ? NB : 0; }

__host__ __device__ inline SmemLayout smem_layout(int NB, int C, int rows_b) {
  SmemLayout s;
  s.a = 0;
  s.ac = al1k(s.a + (size_t)RA * C * 2);
  s.bv = al1k(s.ac + (size_t)(8 + staged_x_rows(NB)) * C * 2);
  const size_t b_bytes = (size_t)RWKV_RANK_SUM * 128 + al1k((size_t)rows_b * 128);
  const size_t v_bytes = (size_t)C * 64;
  s.bc = al1k(s.bv + (b_bytes > v_bytes ? b_bytes : v_bytes));
  s.k = al1k(s.bc + 8 * 128);
  s.cc = al1k(s.k + (size_t)FROWS * C * 2);
  // for NB <= 2 the C-vector region doubles as the [NB][C] fp32 staging of the FFN
  // value sums ((3 + NB) C halves >= NB C floats); four sequences stage them in the
  // consumed FFN key rows
  s.xc = al1k(s.cc + (size_t)(3 + staged_x_rows(NB)) * C * 2);
  s.xr = al1k(s.xc + (size_t)NB * mld_of(C) * 2);
  s.total = al1k(s.xr + (size_t)NB * C * 2);
  return s;
}

// ---- device helpers: timer, barrier, mbarrier, bulk copies, tensor-core tiles
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Grid barrier on a monotonic arrival counter (zeroed before every launch): each CTA
// adds 1 with release semantics and waits, with acquire loads, until the count
// reaches target = (barriers passed so far) x (CTAs). Thread 0 runs `issue` (the next
// phases' bulk copies) between its arrival and its wait, off the critical path.
// Returns false when aborted.
template <typename Issue>
__device__ __forceinline__ bool grid_sync(GridBar* bar, unsigned target, int* s_ok, Issue&& issue) {
  // this thread's generic shared-memory writes before any later bulk copy into them
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&bar->count) : "memory");
    issue();
    if (ld_acquire(&bar->count) < target) {
      const uint64_t t0 = globaltimer();
      unsigned it = 0;
      while (ld_acquire(&bar->count) < target) {
        if ((++it & 63u) == 0) {
          if (ld_relaxed(&bar->abort)) { ok = 0; break; }
          if (globaltimer() - t0 > WAIT_NS) {
            atomicExch(&g_persist_timeout, 1);
            atomicExch(&bar->abort, 1u);
            ok = 0;
            break;
          }
        }
      }
    }
    *s_ok = ok;
  }
  __syncthreads();
  return *s_ok != 0;
}

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for phase `parity` of b; false (error flag + abort word) on expiry.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, GridBar* bar) {
  if (mbar_try_wait(b, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(b, parity)) {
    if (globaltimer() - t0 > WAIT_NS) {
      atomicExch(&g_persist_timeout, 1);
      atomicExch(&bar->abort, 1u);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          saddr(dst)),
      "l"(src), "r"(bytes), "r"(saddr(b))
      : "memory");
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* b) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(saddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(saddr(b)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                       uint64_t* b) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(saddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(saddr(b)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// d (16 x 8, fp32) += a (16 x 16 fp16, row-major) . b (16 x 8 fp16, column-major)
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Staged weight tile, 128B swizzle: element (r, k) of a box of R rows per 64-column
// block at block (k / 64), row r, 16-byte chunk ((k / 8) % 8) ^ (r % 8).
__device__ __forceinline__ uint32_t sw128(uint32_t base, int R, int r, int k) {
  return base + (uint32_t)((((k >> 6) * R + r) << 7) + ((((k >> 3) & 7) ^ (r & 7)) << 4));
}
// ldmatrix x4 lane address of the 16 x 16 A tile at (r0, k0) (matrices: rows +0/+8 x
// columns +0/+8, in a0..a3 order).
__device__ __forceinline__ uint32_t a_tile_addr(uint32_t base, int R, int r0, int k0, int lane) {
  return sw128(base, R, r0 + (lane & 7) + ((lane >> 3) & 1) * 8, k0 + (lane >> 4) * 8);
}
// B operand of sequence n = lane / 4 (zero past NB): x[n][k0 + 2 (lane % 4) ...] and +8.
template <int NB>
__device__ __forceinline__ void b_frag(const __half* x, int ld, int k0, int lane, uint32_t& b0,
                                       uint32_t& b1) {
  const int n = lane >> 2, t = lane & 3;
  if (n < NB) {
    b0 = *reinterpret_cast<const uint32_t*>(x + (size_t)n * ld + k0 + 2 * t);
    b1 = *reinterpret_cast<const uint32_t*>(x + (size_t)n * ld + k0 + 8 + 2 * t);
  } else {
    b0 = b1 = 0u;
  }
}
// D[row][n] of one 16 x 8 tile into st[n * ld + r0 + row] (n < NB).
template <int NB>
__device__ __forceinline__ void stage_tile(float* st, int ld, int r0, const float (&d)[4], int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int n = 2 * t + (e & 1);
    if (n < NB) st[n * ld + r0 + g + (e >> 1) * 8] = d[e];
  }
}
// 32-row x C GEMV on the tensor cores: warp w takes rows 16 (w & 1) .. + 15 and
// columns [(w >> 1) C / 4, ...), two accumulator chains; partials to part[kq][row][n].
template <int NB>
__device__ __forceinline__ void gemv32_partial(uint32_t wbase, int R, const __half* x, int ld,
                                               int C, int warp, int lane, float* part) {
  const int mt = warp & 1, kq = warp >> 1, span = C / 4, kb = kq * span;
  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = kb; k0 < kb + span; k0 += 32) {
    uint32_t a[4], a2[4], b0, b1, b2, b3;
    ldsm_x4(a_tile_addr(wbase, R, 16 * mt, k0, lane), a);
    ldsm_x4(a_tile_addr(wbase, R, 16 * mt, k0 + 16, lane), a2);
    b_frag<NB>(x, ld, k0, lane, b0, b1);
    b_frag<NB>(x, ld, k0 + 16, lane, b2, b3);
    mma16816(d0, a, b0, b1);
    mma16816(d1, a2, b2, b3);
  }
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int row = 16 * mt + g + (e >> 1) * 8, n = 2 * t + (e & 1);
    if (n < NB) part[(kq * 32 + row) * NB + n] = d0[e] + d1[e];
  }
}

__device__ __forceinline__ float ldcg_h(const __half* p) { return __half2float(__ldcg(p)); }

// Four consecutive fp16 channels <-> floats (8-byte accesses).
__device__ __forceinline__ void ld4h(const __half* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void st4h(__half* p, const float (&v)[4]) {
  uint2 u;
  *reinterpret_cast<__half2*>(&u.x) = __floats2half2_rn(v[0], v[1]);
  *reinterpret_cast<__half2*>(&u.y) = __floats2half2_rn(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = u;
}
__device__ __forceinline__ void ldcg4h(const __half* p, float (&v)[4]) {
  const uint2 u = __ldcg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void cp4h(__half* dst, const __half* src) {
  *reinterpret_cast<uint2*>(dst) = __ldcg(reinterpret_cast<const uint2*>(src));
}
// fp16(sum of the NREP fixed-point accumulator replicas) of four channels.
__device__ __forceinline__ void ld_acc_rep(const long long* a, size_t rep_stride, float (&v)[4]) {
  long long s[4] = {0, 0, 0, 0};
#pragma unroll
  for (int r = 0; r < NREP; ++r) {
    const longlong2 t0 = __ldcg(reinterpret_cast<const longlong2*>(a + r * rep_stride));
    const longlong2 t1 = __ldcg(reinterpret_cast<const longlong2*>(a + r * rep_stride + 2));
    s[0] += t0.x; s[1] += t0.y; s[2] += t1.x; s[3] += t1.y;
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = r16(fx_val(s[k]));
}

// Per-CTA staging state: one mbarrier per stream, and how many phases of each were
// issued / consumed (so that an aborting CTA can drain what is still in flight).
enum { MB_A = 0, MB_B, MB_K, MB_V, MB_H0, MB_H1, MB_H2, MB_N };

struct Stage {
  uint64_t* mb;  // [MB_N] in shared memory
  uint32_t issued[MB_N], waited[MB_N];
};

// Every thread waits on the mbarrier (the copies' data is then visible to it); the
// verdict is made uniform across the CTA.
__device__ __forceinline__ bool stage_wait(Stage& s, int i, GridBar* bar) {
  const bool ok = mbar_wait(&s.mb[i], s.waited[i] & 1, bar);
  ++s.waited[i];
  return __syncthreads_and(ok) != 0;
}

__device__ __forceinline__ void stage_drain(Stage& s, GridBar* bar) {
  for (int i = 0; i < MB_N; ++i)
    for (; s.waited[i] < s.issued[i]; ++s.waited[i]) mbar_wait(&s.mb[i], s.waited[i] & 1, bar);
}

// Phase A: the task's RA rows (one 3-D box: [C/64][RA][64], swizzled) and ln1_w |
// ln1_b | mix6 | the sequences' tmix state x rows. Thread 0 only.
__device__ __forceinline__ void stage_a(const PParams& P, const DecLayer& L, const LayerMaps& M,
                                        const __half* tmix_x, const int* s_slot, int NB,
                                        __half* sA, __half* sAc, int cta, uint64_t* mb) {
  const int C = P.C;
  const uint32_t row = (uint32_t)C * 2;
  const bool task = cta < P.n_atask;
  mbar_expect_tx(mb, (task ? (uint32_t)RA * row : 0u) + (uint32_t)(8 + staged_x_rows(NB)) * row);
  if (task) {
    const ATask t = P.atask[cta];
    tma_3d(sA, t.src == 0 ? &M.w_rkv : &M.lora_dn, 0, t.row0, 0, mb);
  }
  bulk_g2s(sAc, L.ln1_w, row, mb);
  bulk_g2s(sAc + C, L.ln1_b, row, mb);
  bulk_g2s(sAc + 2 * C, L.mix6, 6 * row, mb);
  for (int b = 0; b < staged_x_rows(NB); ++b)
    bulk_g2s(sAc + (size_t)(8 + b) * C, tmix_x + (size_t)s_slot[b] * C, row, mb);
  for (int b = staged_x_rows(NB); b < NB; ++b) l2_prefetch_bulk(tmix_x + (size_t)s_slot[b] * C, row);
}

// Phase B: the head's LoRA-up slice [288][64], the CTA's rows of W_o[:, head] (both
// 128-byte swizzle) and the head's eight per-channel vectors (w0 a0 v0 k_k k_a r_k
// lnx_w lnx_b). Thread 0 only.
__device__ __forceinline__ void stage_b(const PParams& P, const DecLayer& L, const LayerMaps& M,
                                        __half* sLU, __half* sWo, __half* sBc, int hc, int c0,
                                        bool work, uint64_t* mb) {
  if (!work) {
    mbar_arrive(mb);
    return;
  }
  mbar_expect_tx(mb, (uint32_t)RWKV_RANK_SUM * 128 + (uint32_t)P.rows_b * 128 + 8 * 128);
  tma_2d(sLU, &M.lora_up, hc, 0, mb);
  tma_2d(sLU + 144 * 64, &M.lora_up, hc, 144, mb);
  tma_2d(sWo, &M.w_o, hc, c0, mb);
  bulk_g2s(sBc + 0 * 64, L.w0 + hc, 128, mb);
  bulk_g2s(sBc + 1 * 64, L.a0 + hc, 128, mb);
  bulk_g2s(sBc + 2 * 64, L.v0 + hc, 128, mb);
  bulk_g2s(sBc + 3 * 64, L.k_k + hc, 128, mb);
  bulk_g2s(sBc + 4 * 64, L.k_a + hc, 128, mb);
  bulk_g2s(sBc + 5 * 64, L.r_k + hc, 128, mb);
  bulk_g2s(sBc + 6 * 64, L.lnx_w + hc, 128, mb);
  bulk_g2s(sBc + 7 * 64, L.lnx_b + hc, 128, mb);
}

// Phase C: the CTA's FFN key rows (one 3-D box: [C/64][FROWS][64], swizzled) and
// ln2_w | ln2_b | ffn_x_k | the sequences' cmix state x rows. Thread 0 only.
__device__ __forceinline__ void stage_k(const PParams& P, const DecLayer& L, const LayerMaps& M,
                                        const __half* cmix_x, const int* s_slot, int NB,
                                        __half* sFk, __half* sCc, int j0, uint64_t* mb) {
  const int C = P.C;
  const uint32_t row = (uint32_t)C * 2;
  mbar_expect_tx(mb, (uint32_t)FROWS * row + (uint32_t)(3 + staged_x_rows(NB)) * row);
  tma_3d(sFk, &M.w_fk, 0, j0, 0, mb);
  bulk_g2s(sCc, L.ln2_w, row, mb);
  bulk_g2s(sCc + C, L.ln2_b, row, mb);
  bulk_g2s(sCc + 2 * C, L.ffn_x_k, row, mb);
  for (int b = 0; b < staged_x_rows(NB); ++b)
    bulk_g2s(sCc + (size_t)(3 + b) * C, cmix_x + (size_t)s_slot[b] * C, row, mb);
  for (int b = staged_x_rows(NB); b < NB; ++b) l2_prefetch_bulk(cmix_x + (size_t)s_slot[b] * C, row);
}

// Phase C: the FFN value slice W_fv[:, j0 : j0 + 32] as [C][32] (64-byte swizzle;
// columns past the CTA's own are multiplied by zero). Thread 0 only.
__device__ __forceinline__ void stage_v(const PParams& P, const LayerMaps& M, __half* sV, int j0,
                                        uint64_t* mb) {
  mbar_expect_tx(mb, (uint32_t)P.C * 64);
  for (int y = 0; y < P.C; y += 256) tma_2d(sV + (size_t)y * 32, &M.w_fv, j0, y, mb);
}

// Head tile i of this CTA's rows [v0, v1): 32 rows (one 3-D box, rows past V read as
// zero), or a bare arrival when the CTA has no such tile. Thread 0 only.
__device__ __forceinline__ void stage_head(const PParams& P, int i, int v0, int v1, __half* dst,
                                           uint64_t* mb) {
  if (v0 + 32 * i >= v1) {
    mbar_arrive(mb);
    return;
  }
  mbar_expect_tx(mb, (uint32_t)32 * P.C * 2);
  tma_3d(dst, &P.head_map, 0, v0 + 32 * i, 0, mb);
}

template <int NB, int CPL>
__global__ void __launch_bounds__(NT, 1) k_dec_persist(const __grid_constant__ PParams P) {
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ float red[32 * 2 * NB];
  __shared__ float part[4 * 32 * NB];  // k-quarter partials of a 32-row GEMV
  constexpr int HLD = FROWS + 8;
  __shared__ __align__(16) __half hh[NB * HLD];  // relu^2 of the FFN key rows
  __shared__ int s_ok;
  __shared__ int s_slot[NB];
  __shared__ int64_t s_tok[NB];
  __shared__ __align__(8) uint64_t s_mb[MB_N];
  const int C = P.C, B = P.B, H = P.H, G = gridDim.x, cta = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int MLD = mld_of(C);
  const SmemLayout lay = smem_layout(NB, C, P.rows_b);
  __half* sA = reinterpret_cast<__half*>(smem + lay.a);
  __half* sAc = reinterpret_cast<__half*>(smem + lay.ac);
  __half* sLU = reinterpret_cast<__half*>(smem + lay.bv);
  __half* sWo = sLU + RWKV_RANK_SUM * 64;  // 1024-aligned: 288 * 128 B = 36 KB
  __half* sV = reinterpret_cast<__half*>(smem + lay.bv);
  __half* sBc = reinterpret_cast<__half*>(smem + lay.bc);
  __half* sFk = reinterpret_cast<__half*>(smem + lay.k);
  __half* sCc = reinterpret_cast<__half*>(smem + lay.cc);
  __half* sXc = reinterpret_cast<__half*>(smem + lay.xc);  // [NB][MLD]
  __half* sXr = reinterpret_cast<__half*>(smem + lay.xr);  // residual stream x [NB][C]
  constexpr int E = 4;   // element-wise channels per thread: c0 = 4 tid .. + 3
  const int c0 = 4 * tid;
  const bool ew = c0 < C;  // threads past C / 4 hold zeros in the LayerNorms
  __half* mix = sFk;                                       // phase A: [6][NB][MLD]
  unsigned char* bscr = smem + lay.a;                      // phase B scratch
  // head tiles (32 rows x C, 64 KB at C = 1024): A rows + A vectors | FFN key rows |
  // B slice / FFN value slice
  auto head_slot = [&](int sl) -> __half* {
    return reinterpret_cast<__half*>(smem + (sl == 0 ? lay.a : (sl == 1 ? lay.k : lay.bv)));
  };
  const size_t BC = (size_t)B * C;
  unsigned target = 0;  // grid barrier arrivals expected so far

  // ---- this CTA's share of every phase
  const bool atask = cta < P.n_atask;
  const int hb = cta / P.gph, jb = cta % P.gph;
  const bool bwork = hb < H;
  const int hc = bwork ? hb * RWKV_HD : 0;
  const int b_c0 = min(C, jb * P.rows_b), b_c1 = min(C, b_c0 + P.rows_b);
  const int ngrp = 4 * C / 8;
  const int f_j0 = 8 * (cta * ngrp / G), f_nj = 8 * ((cta + 1) * ngrp / G) - f_j0;
  const int v0 = min(P.V, cta * P.per_v), v1 = min(P.V, v0 + P.per_v);

  Stage S;
  S.mb = s_mb;
#pragma unroll
  for (int i = 0; i < MB_N; ++i) S.issued[i] = S.waited[i] = 0;
  if (tid < NB) {
    const int b = tid < B ? tid : 0;
    s_slot[tid] = P.slots ? P.slots[b] : P.slot_base + b;
    s_tok[tid] = P.tokens[b];
  }
  if (tid == 0) {
    for (int i = 0; i < MB_N; ++i) mbar_init(&s_mb[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0) {
    stage_a(P, P.layers[0], P.maps[0], P.tmix_x, s_slot, NB, sA, sAc, cta, &s_mb[MB_A]);
    stage_b(P, P.layers[0], P.maps[0], sLU, sWo, sBc, hc, b_c0, bwork, &s_mb[MB_B]);
  }
  ++S.issued[MB_A];
  ++S.issued[MB_B];

  float2 s_pre[NB][8];  // the head's state rows (phase B), loaded before A -> B
  bool alive = true;

  for (int l = 0; l < P.L && alive; ++l) {
    const DecLayer& Lw = P.layers[l];
    long long* acc1 = P.acc + (size_t)l * (1 + NREP) * BC;
    long long* acc2 = acc1 + BC;
    float* rnn = P.rnn + (size_t)l * P.n_slots * H * 4096;
    __half* tmix_x = P.tmix_x + (size_t)l * P.n_slots * C;
    __half* cmix_x = P.cmix_x + (size_t)l * P.n_slots * C;

    // =================== phase A ===================
    {
      float lw[E] = {}, lb[E] = {}, mu[6][E] = {}, x[NB][E], prev[NB][E] = {};
      const long long* acc2p = acc1 - (size_t)NREP * BC;  // previous layer's FFN sums
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const int bb = b < B ? b : 0;
        if (!ew) {
#pragma unroll
          for (int k = 0; k < E; ++k) x[b][k] = 0.f;
        } else if (l == 0) {
          ld4h(P.emb + (size_t)s_tok[b] * C + c0, x[b]);
        } else {
          float xr[E], a[E];
          ld_acc_rep(acc2p + (size_t)bb * C + c0, BC, a);
          ld4h(sXr + (size_t)bb * C + c0, xr);
#pragma unroll
          for (int k = 0; k < E; ++k) x[b][k] = r16(xr[k] + a[k]);
        }
      }
      if (ew)  // unstaged token-shift rows (four-sequence layout), L2-prefetched
        for (int b = staged_x_rows(NB); b < NB; ++b)
          ldcg4h(tmix_x + (size_t)s_slot[b] * C + c0, prev[b]);
      if (l == 10) STAMP(200);
      if (!stage_wait(S, MB_A, P.bar)) { alive = false; break; }
      if (l == 10) STAMP(201);
      if (ew) {
        ld4h(sAc + c0, lw);
        ld4h(sAc + C + c0, lb);
#pragma unroll
        for (int t = 0; t < 6; ++t) ld4h(sAc + (2 + t) * C + c0, mu[t]);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          if (b < staged_x_rows(NB)) ld4h(sAc + (8 + b) * C + c0, prev[b]);
          st4h(sXr + (size_t)b * C + c0, x[b]);  // this layer's input, kept for phase C
        }
        if (cta == 0 && l > 0)  // previous layer's cmix state x (read there by every CTA)
          for (int b = 0; b < B; ++b)
            cp4h(P.cmix_x + (size_t)(l - 1) * P.n_slots * C + (size_t)s_slot[b] * C + c0,
                 P.xln2 + (size_t)b * C + c0);
      }
      if (l == 10) STAMP(203);
      ln_regs<NB, E>(x, lw, lb, C, red);
      if (l == 10) STAMP(204);
      // mixes (lerp.py:106-114: diff in fp16, fused fp16 fma)
      if (ew) {
#pragma unroll
        for (int b = 0; b < NB; ++b) {
#pragma unroll
          for (int t = 0; t < 6; ++t) {
            float m[E];
#pragma unroll
            for (int k = 0; k < E; ++k) m[k] = x[b][k] + mu[t][k] * r16(prev[b][k] - x[b][k]);
            st4h(mix + ((size_t)t * NB + b) * MLD + c0, m);
          }
          if (cta == 0 && b < B) st4h(P.xln1 + (size_t)b * C + c0, x[b]);
        }
      }
      __syncthreads();
      if (l == 10) STAMP(202);
      if (atask) {  // the task's rows on the tensor cores, k-quarter partials summed in order
        const ATask tk = P.atask[cta];
        gemv32_partial<NB>(saddr(sA), RA, mix + (size_t)tk.mix * NB * MLD, MLD, C, warp, lane, part);
        __syncthreads();
        for (int i = tid; i < tk.nrows * NB; i += NT) {
          const int row = i / NB, n = i % NB;
          if (n >= B) continue;
          const float v = ((part[row * NB + n] + part[(32 + row) * NB + n]) +
                           part[(64 + row) * NB + n]) + part[(96 + row) * NB + n];
          const int r = tk.row0 + row;
          if (tk.src == 0) P.rkv[((size_t)(r / C) * B + n) * C + (r % C)] = f2h(v);
          else P.ranks[(size_t)n * RWKV_RANK_SUM + r] = f2h(v);
        }
      }
    }
    if (l == 10) STAMP(205);
    {  // the head's state rows: phase B's CTA jb = 0 overwrites them
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const float* S0 = rnn + ((size_t)s_slot[b] * H + (bwork ? hb : 0)) * 4096;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          s_pre[b][j] = *reinterpret_cast<const float2*>(S0 + (8 * warp + j) * 64 + 2 * lane);
      }
    }
    STAMP(6 * l + 0);
    ++S.issued[MB_K];
    if (!grid_sync(P.bar, target += G, &s_ok, [&] {
          stage_k(P, Lw, P.maps[l], cmix_x, s_slot, NB, sFk, sCc, f_j0, &s_mb[MB_K]);
        })) {
      alive = false;
      break;
    }
    STAMP(6 * l + 1);

    // =================== phase B ===================
    if (l == 10) STAMP(144);
    if (!stage_wait(S, MB_B, P.bar)) { alive = false; break; }
    if (l == 10) STAMP(145);
    if (bwork) {
      constexpr int SLD = RWKV_RANK_SUM + 8;
      __half* srh = reinterpret_cast<__half*>(bscr);  // activated ranks, fp16 hi [NB][SLD]
      __half* srl = srh + NB * SLD;                     // and lo (tanh / sigmoid ranks)
      float* vec = reinterpret_cast<float*>(srl + NB * SLD);  // [7][NB][64]: r w k v A B g
      float* ybuf = vec + 7 * NB * 64;                        // [64]
      float* lora = ybuf + 64;                                // [4][NB][64]: v w a g 12
      __half* ygh = reinterpret_cast<__half*>(lora + 4 * NB * 64);  // [NB][72]
      float* pst = reinterpret_cast<float*>(ygh + NB * 72);          // [NB][128] projection
      auto bvec = [&](int v) {
        return __half22float2(*reinterpret_cast<const __half2*>(sBc + v * 64 + 2 * lane));
      };
      const float2 RK = bvec(5), LW = bvec(6), LB = bvec(7);
      // gate inputs: thread (sequence gb, channel gc) of this head; all of this phase's
      // L2 reads are issued before any of them is used
      const int gb = tid >> 6, gc = tid & 63;
      float r_in = 0.f, k_in = 0.f, v_in = 0.f, vf_in = 0.f;
      if (gb < B) {
        const size_t o = (size_t)gb * C + hc + gc;
        r_in = ldcg_h(P.rkv + o);
        k_in = ldcg_h(P.rkv + BC + o);
        v_in = ldcg_h(P.rkv + 2 * BC + o);
        if (l > 0) vf_in = ldcg_h(P.vfirst + o);
      }
      // activated ranks (gates.py:166-181: tanh for w, sigmoid for g, fp32), split into
      // fp16 hi + lo so that the tensor cores see them to ~22 bits. One or two sequences:
      // every rank load issued before the first is used (measured: B = 1 and 2 gain, the
      // four-sequence layout loses)
      auto act_store = [&](int i, float v) {
        const int b = i / RWKV_RANK_SUM, j = i % RWKV_RANK_SUM;
        if (j >= 32 && j < 96) v = tanhf(v);
        else if (j >= 160) v = sigmoidf_(v);
        const __half hi = f2h(v);
        srh[b * SLD + j] = hi;
        srl[b * SLD + j] = f2h(v - h2f(hi));
      };
      auto ld_rank = [&](int i) {
        const int b = i / RWKV_RANK_SUM, j = i % RWKV_RANK_SUM;
        return b < B ? ldcg_h(P.ranks + (size_t)b * RWKV_RANK_SUM + j) : 0.f;
      };
      if constexpr (NB <= 2) {
        constexpr int RIT = (NB * RWKV_RANK_SUM + NT - 1) / NT;
        float rv[RIT];
#pragma unroll
        for (int u = 0; u < RIT; ++u) {
          const int i = tid + u * NT;
          rv[u] = i < NB * RWKV_RANK_SUM ? ld_rank(i) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < RIT; ++u)
          if (tid + u * NT < NB * RWKV_RANK_SUM) act_store(tid + u * NT, rv[u]);
      } else {
        for (int i = tid; i < NB * RWKV_RANK_SUM; i += NT) act_store(i, ld_rank(i));
      }
      __syncthreads();
      if (l == 10) STAMP(146);
      // LoRA up on the tensor cores: D[c][n] = sum_j W_up[j][c] s[n][j] per gate; warp
      // w takes channels 16 (w % 4) .. + 15; warps 0-3 gates v, w, a, warps 4-7 gate g
      {
        const int c0 = 16 * (warp & 3);
        const uint32_t ub = saddr(sLU);
        // A^T tiles from the [j][c] staging (ldmatrix .trans): lane rows j, chunk of c
        auto a_up = [&](int j0, uint32_t (&a)[4]) {
          const int mi = lane >> 3, j = j0 + (lane & 7) + (mi >> 1) * 8, ch = (c0 >> 3) + (mi & 1);
          ldsm_x4_t(ub + (uint32_t)((j << 7) + ((ch ^ (j & 7)) << 4)), a);
        };
        auto gate = [&](int g, int j_lo, int j_hi, bool split) {
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          for (int j0 = j_lo; j0 < j_hi; j0 += 16) {
            uint32_t a[4], b0, b1;
            a_up(j0, a);
            b_frag<NB>(srh, SLD, j0, lane, b0, b1);
            mma16816(d, a, b0, b1);
            if (split) {
              b_frag<NB>(srl, SLD, j0, lane, b0, b1);
              mma16816(d, a, b0, b1);
            }
          }
          const int gg = lane >> 2, t = lane & 3;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c = c0 + gg + (e >> 1) * 8, n = 2 * t + (e & 1);
            if (n < NB) lora[(g * NB + n) * 64 + c] = d[e];
          }
        };
        if (warp < 4) {
          gate(0, 0, 32, false);
          gate(1, 32, 96, true);
          gate(2, 96, 160, false);
        } else {
          gate(3, 160, 288, true);
        }
      }
      __syncthreads();
      if (l == 10) STAMP(147);
      // gate math + L2 norm, thread (gb, gc) (decode semantics, gates.py:182-213,
      // dplr.py:45-71); the 64-channel sum of kk^2 spans the sequence's two warps
      {
        float kk = 0.f, a16 = 0.f;
        if (gb < B) {
          const float w0 = h2f(sBc[gc]), a0 = h2f(sBc[64 + gc]), v0 = h2f(sBc[128 + gc]);
          const float k_k = h2f(sBc[192 + gc]), k_a = h2f(sBc[256 + gc]);
          float vo;
          if (l == 0) {
            vo = v_in;
            if (jb == 0) P.vfirst[(size_t)gb * C + hc + gc] = f2h(v_in);
          } else {
            vo = r16(v_in + sigmoidf_(v0 + lora[(0 * NB + gb) * 64 + gc]) * (vf_in - v_in));
          }
          const float wd =
              r16(expf(-sigmoidf_(w0 + lora[(1 * NB + gb) * 64 + gc]) / 1.6487212707001282f));
          const float a = sigmoidf_(a0 + lora[(2 * NB + gb) * 64 + gc]);
          a16 = r16(a);
          kk = r16(k_in * k_k);
          const float ko = r16(k_in + k_a * (k_in * a - k_in));
          const int o = gb * 64 + gc;
          vec[0 * NB * 64 + o] = r_in;
          vec[1 * NB * 64 + o] = wd;
          vec[2 * NB * 64 + o] = ko;
          vec[3 * NB * 64 + o] = vo;
          vec[6 * NB * 64 + o] = r16(lora[(3 * NB + gb) * 64 + gc]);
        }
        const float ss = warp_sum(kk * kk);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (gb < B) {
          const float den = fmaxf(sqrtf(red[2 * gb] + red[2 * gb + 1]), 1e-12f);
          const float kn = kk / den;
          const int o = gb * 64 + gc;
          vec[4 * NB * 64 + o] = r16(kn);
          vec[5 * NB * 64 + o] = r16(-(kn * a16));
        }
        if (tid >= B * 64 && tid < NB * 64) ygh[(tid >> 6) * 72 + (tid & 63)] = __float2half(0.f);
      }
      __syncthreads();
      if (l == 10) STAMP(148);
      // wkv7 step per sequence: warp w owns state rows 8w..8w+7, lane columns 2l, 2l+1
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b >= B) break;
        float* Sh = rnn + ((size_t)s_slot[b] * H + hb) * 4096;
        const float* vb = vec + b * 64;
        const float2 rr = make_float2(vb[0 * NB * 64 + 2 * lane], vb[0 * NB * 64 + 2 * lane + 1]);
        const float2 ww = make_float2(vb[1 * NB * 64 + 2 * lane], vb[1 * NB * 64 + 2 * lane + 1]);
        const float2 kk = make_float2(vb[2 * NB * 64 + 2 * lane], vb[2 * NB * 64 + 2 * lane + 1]);
        const float2 aa = make_float2(vb[4 * NB * 64 + 2 * lane], vb[4 * NB * 64 + 2 * lane + 1]);
        const float2 bbv = make_float2(vb[5 * NB * 64 + 2 * lane], vb[5 * NB * 64 + 2 * lane + 1]);
        float2 st[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) st[j] = s_pre[b][j];
        float p[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) p[j] = st[j].x * aa.x + st[j].y * aa.y;
        const float sa_mine = reduce8(p, lane);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float sa = __shfl_sync(0xffffffffu, sa_mine, 4 * j);
          const float v = vb[3 * NB * 64 + 8 * warp + j];
          st[j].x = st[j].x * ww.x + sa * bbv.x + v * kk.x;
          st[j].y = st[j].y * ww.y + sa * bbv.y + v * kk.y;
          if (jb == 0) *reinterpret_cast<float2*>(Sh + (8 * warp + j) * 64 + 2 * lane) = st[j];
          p[j] = st[j].x * rr.x + st[j].y * rr.y;
        }
        const float y_mine = reduce8(p, lane);
        if ((lane & 3) == 0) ybuf[8 * warp + ((lane >> 2) & 7)] = r16(y_mine);
        __syncthreads();
        if (warp == 0) {  // GroupNorm (eps 64e-5) + bonus (dplr.py:73-124), then * g
          const float2 y = make_float2(ybuf[2 * lane], ybuf[2 * lane + 1]);
          const float mean = warp_sum(y.x + y.y) * (1.0f / 64);
          const float dx = y.x - mean, dy = y.y - mean;
          const float var = warp_sum(dx * dx + dy * dy) * (1.0f / 64);
          const float rstd = 1.0f / sqrtf(var + 64e-5f);
          float pr = rr.x * kk.x * RK.x;
          pr += rr.y * kk.y * RK.y;
          const float rkrk = warp_sum(pr);
          const float vx = vb[3 * NB * 64 + 2 * lane], vy = vb[3 * NB * 64 + 2 * lane + 1];
          const float ox = r16(dx * rstd * LW.x + LB.x + rkrk * vx);
          const float oy = r16(dy * rstd * LW.y + LB.y + rkrk * vy);
          *reinterpret_cast<__half2*>(ygh + b * 72 + 2 * lane) =
              __floats2half2_rn(ox * vb[6 * NB * 64 + 2 * lane], oy * vb[6 * NB * 64 + 2 * lane + 1]);
        }
        __syncthreads();
      }
      if (l == 10) STAMP(149);
      // this CTA's rows of the output projection (demo/_rwkv7_base.py:206) on the
      // tensor cores: warp w takes rows 16 w .. + 15 of the W_o slice, K = the head's 64
      {
        const int r0 = 16 * warp;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t ob = saddr(sWo);
#pragma unroll
        for (int k0 = 0; k0 < 64; k0 += 16) {
          uint32_t a[4], b0, b1;
          ldsm_x4(a_tile_addr(ob, 0, r0, k0, lane), a);
          b_frag<NB>(ygh, 72, k0, lane, b0, b1);
          mma16816(d, a, b0, b1);
        }
        stage_tile<NB>(pst, 128, r0, d, lane);
        __syncthreads();
        const int nq = (b_c1 - b_c0) / 4;  // whole quads of rows
        for (int i = tid; i < B * nq; i += NT) {
          const int n = i / nq, q = i % nq;
          const float4 v4 = *reinterpret_cast<const float4*>(pst + n * 128 + 4 * q);
          long long* dst = acc1 + (size_t)n * C + b_c0 + 4 * q;
          fx_add(dst, v4.x); fx_add(dst + 1, v4.y); fx_add(dst + 2, v4.z); fx_add(dst + 3, v4.w);
        }
      }
      if (jb == 0)  // new tmix state x (LN1 output) for this head's channels
        for (int i = tid; i < B * 64; i += NT) {
          const int b = i / 64, c = hc + i % 64;
          tmix_x[(size_t)s_slot[b] * C + c] = __ldcg(P.xln1 + (size_t)b * C + c);
        }
    }
    if (l == 10) STAMP(150);
    // the B slice and scratch are consumed: the FFN value slice and the next layer's A
    // rows (or, in the last layer, head tile 0) take their places
    ++S.issued[MB_V];
    if (l + 1 < P.L) ++S.issued[MB_A];
    else ++S.issued[MB_H0];
    STAMP(6 * l + 2);
    if (!grid_sync(P.bar, target += G, &s_ok, [&] {
          stage_v(P, P.maps[l], sV, f_j0, &s_mb[MB_V]);
          if (l + 1 < P.L)
            stage_a(P, P.layers[l + 1], P.maps[l + 1], P.tmix_x + (size_t)(l + 1) * P.n_slots * C,
                    s_slot, NB, sA, sAc, cta, &s_mb[MB_A]);
          else
            stage_head(P, 0, v0, v1, head_slot(0), &s_mb[MB_H0]);
        })) {
      alive = false;
      break;
    }
    STAMP(6 * l + 3);

    // =================== phase C ===================
    {
      __half* xk = sXc;  // [NB][MLD]
      float lw[E] = {}, lb[E] = {}, mu[E] = {}, x[NB][E], prev[NB][E] = {};
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const int bb = b < B ? b : 0;
        if (ew) {
          float xr[E];
          const longlong2 a01 = __ldcg(reinterpret_cast<const longlong2*>(acc1 + (size_t)bb * C + c0));
          const longlong2 a23 = __ldcg(reinterpret_cast<const longlong2*>(acc1 + (size_t)bb * C + c0 + 2));
          ld4h(sXr + (size_t)bb * C + c0, xr);
          x[b][0] = r16(xr[0] + r16(fx_val(a01.x)));
          x[b][1] = r16(xr[1] + r16(fx_val(a01.y)));
          x[b][2] = r16(xr[2] + r16(fx_val(a23.x)));
          x[b][3] = r16(xr[3] + r16(fx_val(a23.y)));
        } else {
#pragma unroll
          for (int k = 0; k < E; ++k) x[b][k] = 0.f;
        }
      }
      if (ew)
        for (int b = staged_x_rows(NB); b < NB; ++b)
          ldcg4h(cmix_x + (size_t)s_slot[b] * C + c0, prev[b]);
      if (l == 10) STAMP(151);
      if (!stage_wait(S, MB_K, P.bar)) { alive = false; break; }
      if (l == 10) STAMP(152);
      if (ew) {
        ld4h(sCc + c0, lw);
        ld4h(sCc + C + c0, lb);
        ld4h(sCc + 2 * C + c0, mu);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          if (b < staged_x_rows(NB)) ld4h(sCc + (3 + b) * C + c0, prev[b]);
          st4h(sXr + (size_t)b * C + c0, x[b]);  // x1, the next layer's residual
        }
      }
      ln_regs<NB, E>(x, lw, lb, C, red);
      if (ew) {
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          float m[E];
#pragma unroll
          for (int k = 0; k < E; ++k) m[k] = x[b][k] + mu[k] * r16(prev[b][k] - x[b][k]);
          st4h(xk + (size_t)b * MLD + c0, m);
          if (cta == 0 && b < B) st4h(P.xln2 + (size_t)b * C + c0, x[b]);
        }
      }
      __syncthreads();
      if (l == 10) STAMP(153);
      // key rows on the tensor cores: h = relu(fp16(x . Wk))^2 in fp16 (zero past f_nj)
      gemv32_partial<NB>(saddr(sFk), FROWS, xk, MLD, C, warp, lane, part);
      __syncthreads();
      if (tid < NB * FROWS) {
        const int n = tid / FROWS, j = tid % FROWS;
        const float s = ((part[j * NB + n] + part[(32 + j) * NB + n]) + part[(64 + j) * NB + n]) +
                        part[(96 + j) * NB + n];
        const float hv = fmaxf(r16(s), 0.f);
        hh[n * HLD + j] = f2h(j < f_nj ? r16(hv * hv) : 0.f);
      }
      __syncthreads();
      if (NB <= 2 && l + 1 == P.L) {  // key rows consumed: head tile 1 takes their place
        if (tid == 0) stage_head(P, 1, v0, v1, head_slot(1), &s_mb[MB_H1]);
        ++S.issued[MB_H1];
      }
      if (l == 10) STAMP(154);
      if (!stage_wait(S, MB_V, P.bar)) { alive = false; break; }
      if (l == 10) STAMP(155);
      {  // acc2[b][c] += W_fv[c, f_j0 : f_j0 + 32] . h[b] on the tensor cores: warp w
         // takes the 16-row tiles w, w + 8, ...; the slice has a 64-byte swizzle (16-byte
         // chunk q of row c at q ^ ((c / 2) % 4))
        const uint32_t vb = saddr(sV);
        // [NB][C] fp32 staging of the sums: the consumed C vectors, or for four sequences
        // (which do not fit there) the consumed FFN key rows
        float* vst = reinterpret_cast<float*>(NB <= 2 ? sCc : sFk);
        uint32_t hb0[2], hb1[2];
        b_frag<NB>(hh, HLD, 0, lane, hb0[0], hb1[0]);
        b_frag<NB>(hh, HLD, 16, lane, hb0[1], hb1[1]);
        for (int mt = warp; mt < C / 16; mt += 16) {  // tiles mt and mt + 8
          float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
          for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int ks = 0; ks < 2; ++ks) {
              const int r = 16 * (mt + 8 * u) + (lane & 7) + ((lane >> 3) & 1) * 8;
              const int q = 2 * ks + (lane >> 4);
              uint32_t a[4];
              ldsm_x4(vb + (uint32_t)(r * 64 + ((q ^ ((r >> 1) & 3)) << 4)), a);
              mma16816(d[u], a, hb0[ks], hb1[ks]);
            }
          stage_tile<NB>(vst, C, 16 * mt, d[0], lane);
          stage_tile<NB>(vst, C, 16 * (mt + 8), d[1], lane);
        }
        __syncthreads();
        long long* acc2r = acc2 + (size_t)(cta % NREP) * BC;
        for (int i = tid; i < B * C; i += NT) fx_add(acc2r + i, vst[i]);
      }
      if (l + 1 == P.L) {  // the value slice is consumed: head tile 2 takes its place
        __syncthreads();
        if (tid == 0) {
          // four sequences: the key rows held the staged sums until now
          if (NB > 2) stage_head(P, 1, v0, v1, head_slot(1), &s_mb[MB_H1]);
          stage_head(P, 2, v0, v1, head_slot(2), &s_mb[MB_H2]);
        }
        if (NB > 2) ++S.issued[MB_H1];
        ++S.issued[MB_H2];
      }
    }
    STAMP(6 * l + 4);
    if (l + 1 < P.L) ++S.issued[MB_B];
    if (!grid_sync(P.bar, target += G, &s_ok, [&] {
          if (l + 1 < P.L)
            stage_b(P, P.layers[l + 1], P.maps[l + 1], sLU, sWo, sBc, hc, b_c0, bwork, &s_mb[MB_B]);
        })) {
      alive = false;
      break;
    }
    STAMP(6 * l + 5);
  }
  if (!alive) {
    stage_drain(S, P.bar);
    return;
  }

  // =================== head ===================
  // x = x1 + fp16(acc2), ln_out, then logits = head @ x over this CTA's rows, 32-row
  // tiles streamed through three shared-memory slots (tile i in slot i % 3)
  STAMP(250);
  {
    __half* xh = sXc;  // [NB][MLD]
    const long long* acc2 = P.acc + (size_t)(P.L - 1) * (1 + NREP) * BC + BC;
    __half* cmix_last = P.cmix_x + (size_t)(P.L - 1) * P.n_slots * C;
    float lw[E] = {}, lb[E] = {}, x[NB][E];
    if (ew) {
      ld4h(P.lnout_w + c0, lw);
      ld4h(P.lnout_b + c0, lb);
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const int bb = b < B ? b : 0;
      if (ew) {
        float xr[E], a[E];
        ld_acc_rep(acc2 + (size_t)bb * C + c0, BC, a);
        ld4h(sXr + (size_t)bb * C + c0, xr);
#pragma unroll
        for (int k = 0; k < E; ++k) x[b][k] = r16(xr[k] + a[k]);
      } else {
#pragma unroll
        for (int k = 0; k < E; ++k) x[b][k] = 0.f;
      }
    }
    if (cta == 0 && ew)
      for (int b = 0; b < B; ++b) cp4h(cmix_last + (size_t)s_slot[b] * C + c0, P.xln2 + (size_t)b * C + c0);
    ln_regs<NB, E>(x, lw, lb, C, red);
    if (ew)
#pragma unroll
      for (int b = 0; b < NB; ++b) st4h(xh + (size_t)b * MLD + c0, x[b]);
    __syncthreads();
    const int ntile = (v1 - v0 + 31) / 32;
    for (int i = 0; i < ntile; ++i) {
      const int sl = i % 3;
      if (!stage_wait(S, MB_H0 + sl, P.bar)) {
        stage_drain(S, P.bar);
        return;
      }
      gemv32_partial<NB>(saddr(head_slot(sl)), 32, xh, MLD, C, warp, lane, part);
      __syncthreads();  // slot consumed
      if (i + 3 < ntile) {
        if (tid == 0) stage_head(P, i + 3, v0, v1, head_slot(sl), &s_mb[MB_H0 + sl]);
        ++S.issued[MB_H0 + sl];
      }
      for (int j = tid; j < 32 * NB; j += NT) {
        const int row = j / NB, n = j % NB, v = v0 + 32 * i + row;
        if (n < B && v < v1)
          P.logits[(size_t)n * P.V + v] = f2h(((part[row * NB + n] + part[(32 + row) * NB + n]) +
                                               part[(64 + row) * NB + n]) + part[(96 + row) * NB + n]);
      }
      __syncthreads();  // partials read
    }
    stage_drain(S, P.bar);
  }
  STAMP(251);
}

// ---------------------------------------------------------------------------
// host side
int device_sms() {
  static std::mutex mu;
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> g(mu);
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return sms[dev];
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Map key: pointer, rank, shape, box and swizzle.
struct MapKey {
  const void* ptr;
  int rank, rows, cols, box_cols, box_rows, swz, dev;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rank == o.rank && rows == o.rows && cols == o.cols &&
           box_cols == o.box_cols && box_rows == o.box_rows && swz == o.swz && dev == o.dev;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = reinterpret_cast<size_t>(k.ptr);
    h ^= (size_t)k.rows * 0x9E3779B97F4A7C15ull + (size_t)k.cols * 0xC2B2AE3D27D4EB4Full +
         (size_t)k.box_cols * 0x165667B19E3779F9ull + (size_t)k.box_rows * 31 + (size_t)k.swz * 7 +
         (size_t)k.dev * 131 + (size_t)k.rank * 1009;
    return h;
  }
};

// fp16 row-major [rows, cols] tensor map (cached: weights do not move while a model is
// alive). rank 2: box [box_rows, box_cols]; rank 3: 64-column blocks as a third
// dimension, box (64, box_rows, cols / 64), so that one copy lands a row block as
// [cols / 64][box_rows][64]. swz: 0 none, 64 or 128 bytes.
int make_map(CUtensorMap* out, const void* ptr, int rank, int rows, int cols, int box_cols,
             int box_rows, int swz) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const MapKey key{ptr, rank, rows, cols, box_cols, box_rows, swz, dev};
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return RWKV_OK;
  }
  auto fn = encode_fn();
  if (!fn) {
    rwkv_set_error("decode_persist: cuTensorMapEncodeTiled unavailable");
    return RWKV_ERR_CUDA;
  }
  const CUtensorMapSwizzle sw = swz == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swz == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                            : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUtensorMap m;
  CUresult r;
  if (rank == 2) {
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    const cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(cols / 64)};
    const cuuint64_t strides[2] = {(cuuint64_t)cols * 2, 128};
    const cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)(cols / 64)};
    const cuuint32_t estr[3] = {1, 1, 1};
    r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) {
    rwkv_set_error("decode_persist: cuTensorMapEncodeTiled failed (%d) rank=%d rows=%d cols=%d box=%dx%d",
                   (int)r, rank, rows, cols, box_rows, box_cols);
    return RWKV_ERR_CUDA;
  }
  cache.emplace(key, m);
  *out = m;
  return RWKV_OK;
}

int rows_b_of(int C, int G) {
  const int gph = G / (C / RWKV_HD);
  return ((C + gph - 1) / gph + 3) & ~3;
}

// Phase-A tasks: each mix group's rows cut into blocks of <= RA rows (r | k | v rows of
// W_rkv; LoRA v | w | a | g rows of W_lora_dn). Returns the task count (cap + 1 when
// they do not fit).
int build_atasks(int C, ATask* out, int cap) {
  struct Seg {
    int src, row0, rows, mix;
  };
  const Seg segs[7] = {{0, 0, C, 0},  {0, C, C, 2},   {0, 2 * C, C, 3}, {1, 0, 32, 3},
                       {1, 32, 64, 1}, {1, 96, 64, 4}, {1, 160, 128, 5}};
  int n = 0;
  for (const Seg& s : segs)
    for (int r = 0; r < s.rows; r += RA) {
      if (n >= cap) return cap + 1;
      out[n++] = ATask{s.src, s.row0 + r, s.rows - r < RA ? s.rows - r : RA, s.mix};
    }
  return n;
}

}  // namespace

int check_model_public(const rwkv7_model* m);

// Workspace for the persistent path: activations + per-layer accumulators + the grid
// barrier, laid out so one memset clears the accumulators and the barrier together.
struct PersistWork {
  __half *xln1, *xln2, *rkv, *ranks, *vfirst;
  long long* acc;
  GridBar* bar;
  size_t zero_bytes;
};

static size_t carve_persist(void* base, PersistWork* w, int L, int B, int C) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? static_cast<char*>(base) + off : nullptr;
    off += (bytes + 255) & ~size_t(255);
    return p;
  };
  const size_t BC = (size_t)B * C;
  PersistWork d;
  d.xln1 = (__half*)take(BC * 2);
  d.xln2 = (__half*)take(BC * 2);
  d.rkv = (__half*)take(3 * BC * 2);
  d.ranks = (__half*)take((size_t)B * RWKV_RANK_SUM * 2);
  d.vfirst = (__half*)take(BC * 2);
  const size_t acc_off = off;
  d.acc = (long long*)take((size_t)L * (1 + NREP) * BC * 8);
  d.bar = (GridBar*)take(sizeof(GridBar));
  d.zero_bytes = off - acc_off;
  if (w) *w = d;
  return off;
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Whether the persistent path covers this problem on the current device: sizes it was
// laid out for, shared memory, and 16-byte alignment of everything a bulk copy reads.
bool decode_persist_supported(const rwkv7_model* m, int B, const rwkv7_state* state) {
  if (B < 1 || B > PMAXB || m->n_layer > PMAXL) return false;
  if (m->n_embd != 768 && m->n_embd != 1024) return false;
  if (!al16(m->head) || !al16(state->tmix_x) || !al16(state->cmix_x)) return false;
  for (int l = 0; l < m->n_layer; ++l) {
    const rwkv7_layer& s = m->layers[l];
    const void* ptrs[] = {s.w_rkv, s.w_lora_dn, s.w_lora_up, s.ln1_w, s.ln1_b, s.mix6, s.w0,
                          s.a0, s.v0, s.k_k, s.k_a, s.r_k, s.lnx_w, s.lnx_b, s.w_o, s.ln2_w,
                          s.ln2_b, s.ffn_x_k, s.w_fk, s.w_fv};
    for (const void* q : ptrs)
      if (!al16(q)) return false;
  }
  const char* e = std::getenv("RWKV_B200_DECODE_PERSIST");
  if (e && e[0] == '0') return false;
  const int G = device_sms();
  const int C = m->n_embd, H = C / RWKV_HD;
  if (G > MAXG || G < H * 8 || G > 4 * C / 8 || rows_b_of(C, G) > 128) return false;
  ATask tmp[MAXG];
  if (build_atasks(C, tmp, MAXG) > G) return false;
  if ((4 * C / 8 + G - 1) / G > FROWS / 8) return false;
  const int NB = B <= 2 ? B : 4;
  const size_t smem = smem_layout(NB, C, rows_b_of(C, G)).total;
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return smem + 4096 <= (size_t)optin;
}

size_t decode_persist_workspace(const rwkv7_model* m, int B) {
  return carve_persist(nullptr, nullptr, m->n_layer, B, m->n_embd);
}

template <int NB, int CPL>
static int run_persist(const rwkv7_model* m, const int64_t* tokens, int B, const int* slots,
                       int slot_base, const rwkv7_state* state, void* logits, void* ws,
                       cudaStream_t st) {
  const int L = m->n_layer, C = m->n_embd, H = C / RWKV_HD, G = device_sms();
  PersistWork w;
  carve_persist(ws, &w, L, B, C);
  static PParams P;  // ~28 KB: kept off the stack; the launch copies its arguments
  static std::mutex pmu;
  std::lock_guard<std::mutex> lk(pmu);
  P = PParams{};
  P.B = B; P.C = C; P.H = H; P.L = L; P.V = m->vocab; P.n_slots = state->n_slots;
  P.n_atask = build_atasks(C, P.atask, MAXG);
  P.gph = G / H;
  P.rows_b = rows_b_of(C, G);
  P.per_v = (m->vocab + G - 1) / G;
  P.tokens = tokens; P.slots = slots; P.slot_base = slot_base;
  P.emb = (const __half*)m->emb; P.head = (const __half*)m->head;
  P.lnout_w = (const __half*)m->lnout_w; P.lnout_b = (const __half*)m->lnout_b;
  P.logits = (__half*)logits;
  P.xln1 = w.xln1; P.xln2 = w.xln2;
  P.rkv = w.rkv; P.ranks = w.ranks; P.vfirst = w.vfirst; P.acc = w.acc; P.bar = w.bar;
  P.rnn = (float*)state->rnn;
  P.tmix_x = (__half*)state->tmix_x;
  P.cmix_x = (__half*)state->cmix_x;
  for (int l = 0; l < L; ++l) {
    const rwkv7_layer& s = m->layers[l];
    P.layers[l] = {(const __half*)s.ln1_w, (const __half*)s.ln1_b, (const __half*)s.ln2_w,
                   (const __half*)s.ln2_b, (const __half*)s.mix6, (const __half*)s.w_rkv,
                   (const __half*)s.w_lora_dn, (const __half*)s.w_lora_up, (const __half*)s.w0,
                   (const __half*)s.a0, (const __half*)s.v0, (const __half*)s.k_k,
                   (const __half*)s.k_a, (const __half*)s.r_k, (const __half*)s.lnx_w,
                   (const __half*)s.lnx_b, (const __half*)s.w_o, (const __half*)s.ffn_x_k,
                   (const __half*)s.w_fk, (const __half*)s.w_fv};
    LayerMaps& M = P.maps[l];
    int rc;
    if ((rc = make_map(&M.w_rkv, s.w_rkv, 3, 3 * C, C, 64, RA, 128)) ||
        (rc = make_map(&M.lora_dn, s.w_lora_dn, 3, RWKV_RANK_SUM, C, 64, RA, 128)) ||
        (rc = make_map(&M.w_fk, s.w_fk, 3, 4 * C, C, 64, FROWS, 128)) ||
        (rc = make_map(&M.lora_up, s.w_lora_up, 2, RWKV_RANK_SUM, C, 64, 144, 128)) ||
        (rc = make_map(&M.w_o, s.w_o, 2, C, C, 64, P.rows_b, 128)) ||
        (rc = make_map(&M.w_fv, s.w_fv, 2, C, 4 * C, 32, 256, 64)))
      return rc;
  }
  {
    const int rc = make_map(&P.head_map, m->head, 3, m->vocab, C, 64, 32, 128);
    if (rc) return rc;
  }
  const size_t smem = smem_layout(NB, C, P.rows_b).total;
  auto kern = k_dec_persist<NB, CPL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    rwkv_set_error("decode_persist: cudaFuncSetAttribute(%zu B smem): %s", smem, cudaGetErrorString(e));
    return RWKV_ERR_CUDA;
  }
  if (cudaMemsetAsync(w.acc, 0, w.zero_bytes, st) != cudaSuccess)
    return rwkv_check_launch("decode_persist memset");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, P);
  if (e != cudaSuccess) {
    rwkv_set_error("decode_persist: launch failed: %s", cudaGetErrorString(e));
    return RWKV_ERR_CUDA;
  }
  return rwkv_check_launch("decode_persist");
}

// One launch: the one-, two- or four-sequence layout (B = 3 runs the four-sequence
// layout with one column idle).
int decode_persist_run(const rwkv7_model* m, const int64_t* tokens, int B, const int* slots,
                       const rwkv7_state* state, void* logits, void* ws, cudaStream_t st) {
  const bool c768 = m->n_embd == 768;
  if (B == 1) return c768 ? run_persist<1, 3>(m, tokens, 1, slots, 0, state, logits, ws, st)
                          : run_persist<1, 4>(m, tokens, 1, slots, 0, state, logits, ws, st);
  if (B == 2) return c768 ? run_persist<2, 3>(m, tokens, 2, slots, 0, state, logits, ws, st)
                          : run_persist<2, 4>(m, tokens, 2, slots, 0, state, logits, ws, st);
  return c768 ? run_persist<4, 3>(m, tokens, B, slots, 0, state, logits, ws, st)
              : run_persist<4, 4>(m, tokens, B, slots, 0, state, logits, ws, st);
}

#if PERSIST_STAMPS
extern "C" int rwkv7_decode_persist_stamps(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, g_stamp, sizeof(g_stamp)) == cudaSuccess ? 0 : 1;
}
#endif

// Self-test of the persistent kernel's bounded waits, with the same device functions:
// a grid barrier whose target the single CTA can never reach, then an mbarrier that
// nothing arrives on. Both must give up after WAIT_NS, set the device error flag and
// return. `bar` is 16 zeroed bytes of device memory supplied by the caller.
namespace {
__global__ void k_wait_selftest_persist(GridBar* bar, int* out) {
  __shared__ int s_ok;
  __shared__ __align__(8) uint64_t mb;
  const bool grid_ok = grid_sync(bar, 2u, &s_ok, [] {});
  if (threadIdx.x == 0) {
    mbar_init(&mb, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    bar->abort = 0;  // the grid wait raised it; clear so the mbarrier wait runs to its limit
    const bool mb_ok = mbar_wait(&mb, 0, bar);
    out[0] = (grid_ok ? 0 : 1) | (mb_ok ? 0 : 2);
  }
}
}  // namespace
int wait_selftest_persist(void* bar, int* out, cudaStream_t st) {
  return rwkv_launch("wait_selftest_persist", k_wait_selftest_persist, dim3(1), dim3(64), 0, st,
                     static_cast<GridBar*>(bar), out);
}

int decode_persist_timeout_flag() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_persist_timeout, sizeof(int));
  if (v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_persist_timeout, &z, sizeof(int));
  }
  return v;
}
