// Grouped fp16 GEMM on the 5th-generation tensor cores (tcgen05 + TMA + TMEM).
//
// C[M, N] = epi(A[M, K] @ B[N, K]^T): A and B are both K-major (row-major with
// the reduction dim contiguous), which is the layout every projection here
// has (weights keep the checkpoint's [out, in] orientation).
//
// One CTA computes a 128 x BN output tile (or a K-slice of it, split-K):
//   warp 0      TMA producer: 128B-swizzled 128x64 (A) and BNx64 (B) fp16 tiles
//               into a STAGES-deep shared-memory ring (mbarrier full/empty);
//   warp 1      allocates BN TMEM columns, one elected thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) x 4 per
//               stage and tcgen05.commit's the stage back to the producer;
//   warps 2-5   epilogue: tcgen05.ld 32x32b (each warp its 32-lane TMEM
//               quadrant = 32 output rows), fused epilogue, fp16 stores; with
//               split-K each CTA parks its fp32 partial tile and
//               k_splitk_reduce sums the slices in split order (deterministic)
//               and applies the epilogue.
// No TMA multicast is used anywhere (the kernels also run in multi-GPU jobs).
// Every mbarrier wait is bounded: on timeout the CTA records an error flag
// and leaves its loops instead of spinning forever.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "common.cuh"

namespace {

constexpr int BM = 128, BK = 64;
constexpr int NTHREADS = 192;
constexpr uint64_t WAIT_NS = 1000000000ull;  // 1 s: a pipeline barrier gave up

__device__ int g_tc_timeout = 0;

struct TcProblem {
  void* C;
  const void* R;
  float* ws;     // split-K partial tiles [splits][M][N] fp32, or null
  int M, N, K, ldc;
};

struct TcParams {
  CUtensorMap ta[4];
  CUtensorMap tb[4];
  TcProblem p[4];
  int n_problems;
  int splits;
};

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_plain(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(saddr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t tc_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait; false (and the global error flag set) if the phase has not completed
// within WAIT_NS of wall time (the timer is read once per 256 polls).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = tc_globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && tc_globaltimer() - t0 > WAIT_NS) break;
  }
  atomicExch(&g_tc_timeout, 1);
  return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(saddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(saddr(bar)), "r"(x), "r"(y)
      : "memory");
}

// K-major operand tile with 128-byte swizzle: rows of 64 fp16 (128 B), 8-row
// swizzle atoms 1024 B apart (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void* tile) {
  const uint64_t addr = saddr(tile);
  uint64_t d = (addr >> 4) & 0x3FFFull;
  d |= (uint64_t)1 << 16;            // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;            // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;            // SWIZZLE_128B
  return d;
}

// Instruction descriptor: fp16 A/B, fp32 D, both K-major, M = 128, N = BN.
template <int BN>
__device__ __forceinline__ uint32_t instr_desc() {
  return (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  uint32_t m0 = 0, m1 = 0, m2 = 0, m3 = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(m0), "r"(m1), "r"(m2), "r"(m3));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   saddr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
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

// Apply the epilogue to 16 consecutive columns of one output row and store.
template <int EPI>
__device__ __forceinline__ void store16(const float (&v)[16], void* Cv, const __half* R, int row,
                                        int col, int N, int ldc, bool vec, int prob) {
  const size_t o = (size_t)row * ldc + col;
  if (EPI == RWKV_EPI_STORE_F32 && col + 16 <= N && (ldc & 3) == 0 &&
      (reinterpret_cast<uintptr_t>(Cv) & 15) == 0) {
    // four 16-byte stores: the epilogue's cost is per store instruction
    float4* C = reinterpret_cast<float4*>(static_cast<float*>(Cv) + o);
#pragma unroll
    for (int i = 0; i < 4; ++i) C[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    return;
  }
  if (EPI != RWKV_EPI_STORE_F32 && EPI != RWKV_EPI_LORA_ACT2 && col + 16 <= N && vec) {
    __half* C = static_cast<__half*>(Cv);
    uint4 pk[2];
    __half2* h2 = reinterpret_cast<__half2*>(pk);
    __half tmp[2];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      epi_store2<EPI>(tmp, 0, v[2 * i], v[2 * i + 1], R + o + 2 * i, prob);
      h2[i] = *reinterpret_cast<__half2*>(tmp);
    }
    reinterpret_cast<uint4*>(C + o)[0] = pk[0];
    reinterpret_cast<uint4*>(C + o)[1] = pk[1];
  } else {
    for (int i = 0; i + 1 < 16 && col + i < N; i += 2)
      epi_store2<EPI>(Cv, o + i, v[i], v[i + 1], R, prob);
  }
}

template <int BN, int EPI, int STAGES>
__global__ void __launch_bounds__(NTHREADS, 1) k_gemm_tc(const __grid_constant__ TcParams prm) {
  extern __shared__ unsigned char smem_raw[];
  const int g = blockIdx.z % prm.n_problems;
  const int split = blockIdx.z / prm.n_problems;
  const TcProblem& P = prm.p[g];
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  if (n0 >= P.N || m0 >= P.M) {
    grid_dep_wait();
    return;
  }
  const int KB = (P.K + BK - 1) / BK;  // a partial last K-block reads zeros past K (TMA fill)
  const int kb_per = (KB + prm.splits - 1) / prm.splits;
  const int kb0 = split * kb_per, kb1 = min(KB, kb0 + kb_per);
  // a K-slice past the end still writes its (zero) partial tile for the reduce
  const bool no_k = kb0 >= kb1;
  if (no_k && prm.splits == 1) {
    grid_dep_wait();
    return;
  }

  // shared memory: [A stages][B stages] (1024-aligned) | barriers | tmem address
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
  unsigned char* sA = base;
  unsigned char* sB = base + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     saddr(tmem_slot)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      // B (weights, never written by the preceding kernels) of the first stages goes
      // out before the programmatic wait; A (activations) only after it
      const int pre = min(STAGES, kb1 - kb0);
      for (int i = 0; i < pre; ++i) {
        mbar_expect_tx(&full[i], A_BYTES + B_BYTES);
        tma_load_2d(sB + i * B_BYTES, &prm.tb[g], &full[i], (kb0 + i) * BK, n0);
      }
      grid_dep_wait();
      grid_dep_trigger();
      for (int i = 0; i < pre; ++i) tma_load_2d(sA + i * A_BYTES, &prm.ta[g], &full[i], (kb0 + i) * BK, m0);
      int issued = pre;
      for (int kb = kb0 + pre; kb < kb1; ++kb) {
        const int s = issued % STAGES;
        const uint32_t round = issued / STAGES;
        if (!mbar_wait(&empty[s], (round & 1) ^ 1)) break;
        mbar_expect_tx(&full[s], A_BYTES + B_BYTES);
        tma_load_2d(sA + s * A_BYTES, &prm.ta[g], &full[s], kb * BK, m0);
        tma_load_2d(sB + s * B_BYTES, &prm.tb[g], &full[s], kb * BK, n0);
        ++issued;
      }
      // drain: never leave the CTA while copies may still land in shared memory
      for (int i = max(0, issued - STAGES); i < issued; ++i)
        mbar_wait(&full[i % STAGES], (i / STAGES) & 1);
    } else {
      grid_dep_wait();
      grid_dep_trigger();
    }
  } else if (warp == 1) {
    grid_dep_wait();
    grid_dep_trigger();
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = instr_desc<BN>();
      int it = 0;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(&full[s], (it / STAGES) & 1)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t ad = smem_desc_sw128(sA + s * A_BYTES);
        const uint64_t bd = smem_desc_sw128(sB + s * B_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // +32 bytes per K=16 step inside the 128-byte swizzle atom (>> 4 in the descriptor)
          umma_f16(tmem, ad + (uint64_t)(2 * kk), bd + (uint64_t)(2 * kk), idesc,
                   (kb > kb0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      if (kb0 < kb1) {
        umma_commit(tmem_full);
      } else {
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(tmem_full)) : "memory");
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    grid_dep_wait();
    grid_dep_trigger();
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const bool ok = mbar_wait(tmem_full, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int row = m0 + quad * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    void* C = P.C;
    const __half* R = static_cast<const __half*>(P.R);
    const bool vec = (P.ldc & 7) == 0 && (reinterpret_cast<uintptr_t>(C) & 15) == 0;
    const bool all_ok = __all_sync(0xffffffffu, ok);
    if (!P.ws && EPI == EPI_ARGMAX) {
      // greedy lm head: this tile's best (fp16 logit, lowest column) of the row
      if (all_ok) {
        unsigned long long best = 0;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tmem_ld16(trow + c0, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int col = n0 + c0 + i;
            if (col < P.N) {
              const unsigned long long key = argmax_key(r16(v[i]), col);
              best = key > best ? key : best;
            }
          }
        }
        if (row < P.M) atomicMax(static_cast<unsigned long long*>(C) + row, best);
      }
    } else if (!P.ws) {
      if (all_ok) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tmem_ld16(trow + c0, v);  // all lanes execute (sync.aligned)
          const int col = n0 + c0;
          if (row < P.M && col < P.N) store16<EPI>(v, C, R, row, col, P.N, P.ldc, vec, g);
        }
      }
    } else {
      // split-K: park this K-slice's fp32 tile; k_splitk_reduce sums the slices
      if (all_ok) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tmem_ld16(trow + c0, v);
          if (no_k) {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
          }
          const int col = n0 + c0;
          if (row < P.M && col < P.N) {
            float* dst = P.ws + ((size_t)split * P.M + row) * P.N + col;
            if (col + 16 <= P.N && (P.N & 3) == 0) {
#pragma unroll
              for (int i = 0; i < 4; ++i)
                reinterpret_cast<float4*>(dst)[i] =
                    make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            } else {
              for (int i = 0; i < 16 && col + i < P.N; ++i) dst[i] = v[i];
            }
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
  }
}

struct ReduceParams {
  TcProblem p[4];
  int n_problems, splits;
};

// Split-K reduce: C = epi(sum_s ws[s]) for every problem. grid = (ceil(max M*N/4 / 256), n).
template <int EPI>
__global__ void __launch_bounds__(256) k_splitk_reduce(const __grid_constant__ ReduceParams rp) {
  RWKV_GRID_DEP_ENTRY();
  const TcProblem& P = rp.p[blockIdx.y];
  const size_t MN = (size_t)P.M * P.N;
  const size_t i = ((size_t)blockIdx.x * 256 + threadIdx.x) * 4;
  if (i >= MN) return;
  const int row = (int)(i / P.N), col = (int)(i % P.N);  // N % 4 == 0: 4 columns, one row
  float4 acc = __ldcg(reinterpret_cast<const float4*>(P.ws + i));
  for (int s = 1; s < rp.splits; ++s) {
    const float4 q = __ldcg(reinterpret_cast<const float4*>(P.ws + s * MN + i));
    acc.x += q.x; acc.y += q.y; acc.z += q.z; acc.w += q.w;
  }
  const __half* R = static_cast<const __half*>(P.R);
  const size_t o = (size_t)row * P.ldc + col;
  epi_store2<EPI>(P.C, o, acc.x, acc.y, R, blockIdx.y);
  epi_store2<EPI>(P.C, o + 2, acc.z, acc.w, R, blockIdx.y);
}

// ---------------------------------------------------------------------------
// host side: tensor maps (cached), launch
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct MapKey {
  const void* ptr;
  int rows, cols, ld, box_rows, dev;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && ld == o.ld &&
           box_rows == o.box_rows && dev == o.dev;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = reinterpret_cast<size_t>(k.ptr);
    h ^= (size_t)k.rows * 0x9E3779B97F4A7C15ull + (size_t)k.cols * 0xC2B2AE3D27D4EB4Full +
         (size_t)k.ld * 0x165667B19E3779F9ull + (size_t)k.box_rows * 31 + (size_t)k.dev * 7;
    return h;
  }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// 2-D fp16 row-major [rows, cols] (row stride ld elements), box = [box_rows, 64], 128B swizzle.
int make_map(CUtensorMap* out, const void* ptr, int rows, int cols, int ld, int box_rows) {
  int dev = 0;
  cudaGetDevice(&dev);
  const MapKey key{ptr, rows, cols, ld, box_rows, dev};
  {
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return RWKV_OK;
    }
  }
  auto enc = get_encode();
  if (!enc) {
    rwkv_set_error("gemm_tc: cuTensorMapEncodeTiled unavailable");
    return RWKV_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    rwkv_set_error("gemm_tc: cuTensorMapEncodeTiled failed (%d) rows=%d cols=%d ld=%d", (int)r,
                   rows, cols, ld);
    return RWKV_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lk(g_map_mu);
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps.emplace(key, *out);
  return RWKV_OK;
}

template <int BN, int STAGES>
constexpr int smem_bytes() {
  return 1024 + STAGES * (BM * BK * 2 + BN * BK * 2) + (2 * STAGES + 1) * 8 + 16;
}

template <int BN, int EPI, int STAGES>
int launch_tc(const TcParams& prm, dim3 grid, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  static bool done[64] = {};
  if (dev < 64 && !done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<BN, EPI, STAGES>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem_bytes<BN, STAGES>());
    if (e != cudaSuccess) {
      rwkv_set_error("gemm_tc: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return RWKV_ERR_CUDA;
    }
    done[dev] = true;
  }
  return rwkv_launch("gemm_tc", k_gemm_tc<BN, EPI, STAGES>, grid, dim3(NTHREADS),
                     (size_t)smem_bytes<BN, STAGES>(), st, prm);
}

// ---------------------------------------------------------------------------
// Persistent variant for large problems (every N >= 256, enough tiles to fill the
// GPU): one CTA per SM walks 128 x 256 output tiles (M fastest, so CTAs running at
// the same time share weight tiles in L2). An M=128 x K=16 MMA costs nearly the
// same time at N=64, 128 or 256 (measured), so the widest tile does the most math
// per MMA issued. Two 256-column TMEM accumulators let the epilogue warps drain
// tile j while the MMA thread already accumulates tile j+1:
//   tmem_full[b]  MMA -> epilogue  (tcgen05.commit after the tile's last K-block)
//   tmem_empty[b] epilogue -> MMA  (4 arrivals, one per epilogue warp)
// The operand ring (full/empty, PSTAGES deep) runs continuously across tiles.
constexpr int PBN = 256, PSTAGES = 4;

struct TileMap {
  int base[4 + 1];  // first tile of each problem
  int tiles_m[4];
};

__device__ __forceinline__ void tile_of(const TcParams& prm, const TileMap& tm, int t, int& g,
                                        int& m0, int& n0) {
  g = 0;
  while (g + 1 < prm.n_problems && t >= tm.base[g + 1]) ++g;
  const int local = t - tm.base[g];
  m0 = (local % tm.tiles_m[g]) * BM;
  n0 = (local / tm.tiles_m[g]) * PBN;
}

// Epilogue of one 128-row x PBN-column accumulator slice (TMEM lanes quad*32.., columns
// from trow): thread `row` of the output drains its TMEM lane through the fused epilogue.
template <int EPI>
__device__ __forceinline__ void persist_epilogue(const TcProblem& P, int g, int row, int n0,
                                                 uint32_t trow) {
  void* C = P.C;
  const __half* R = static_cast<const __half*>(P.R);
  if constexpr (EPI == EPI_ARGMAX) {
    unsigned long long best = 0;
#pragma unroll 1
    for (int c0 = 0; c0 < PBN; c0 += 16) {
      float v[16];
      tmem_ld16(trow + c0, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int col = n0 + c0 + i;
        if (col < P.N) {
          const unsigned long long key = argmax_key(r16(v[i]), col);
          best = key > best ? key : best;
        }
      }
    }
    if (row < P.M) atomicMax(static_cast<unsigned long long*>(C) + row, best);
  } else {
    const bool vec = (P.ldc & 7) == 0 && (reinterpret_cast<uintptr_t>(C) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(R) & 15) == 0;
    if (EPI == RWKV_EPI_RESID && vec && n0 + PBN <= P.N) {
      // residual rows: fetch the thread's whole 128-column slice first, so the tile
      // pays one memory latency per half instead of one per 16 columns
#pragma unroll 1
      for (int h0 = 0; h0 < PBN; h0 += 128) {
        uint4 rr[16];
        const __half* rp = R + (size_t)row * P.ldc + n0 + h0;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          rr[i] = row < P.M ? *reinterpret_cast<const uint4*>(rp + 8 * i) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int c1 = 0; c1 < 128; c1 += 16) {
          float v[16];
          tmem_ld16(trow + h0 + c1, v);
          if (row < P.M) {
            uint4 pk[2];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const __half2* r2 = reinterpret_cast<const __half2*>(&rr[c1 / 8 + q]);
              __half2* o2 = reinterpret_cast<__half2*>(&pk[q]);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 rf = __half22float2(r2[e]);
                o2[e] = __floats2half2_rn(rf.x + r16(v[8 * q + 2 * e]), rf.y + r16(v[8 * q + 2 * e + 1]));
              }
            }
            __half* cp = static_cast<__half*>(C) + (size_t)row * P.ldc + n0 + h0 + c1;
            reinterpret_cast<uint4*>(cp)[0] = pk[0];
            reinterpret_cast<uint4*>(cp)[1] = pk[1];
          }
        }
      }
    } else {
#pragma unroll 1
      for (int c0 = 0; c0 < PBN; c0 += 16) {
        float v[16];
        tmem_ld16(trow + c0, v);
        const int col = n0 + c0;
        if (row < P.M && col < P.N) store16<EPI>(v, C, R, row, col, P.N, P.ldc, vec, g);
      }
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_gemm_tc_persist(const __grid_constant__ TcParams prm, const __grid_constant__ TileMap tm) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = BM * BK * 2, B_BYTES = PBN * BK * 2;
  unsigned char* sA = base;
  unsigned char* sB = base + PSTAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + PSTAGES * B_BYTES);
  uint64_t* empty = full + PSTAGES;
  uint64_t* tfull = empty + PSTAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  const int total = tm.base[prm.n_problems];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     saddr(tmem_slot)),
                 "r"(2 * PBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int it = 0;
      bool ok = true;
      bool waited = false;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int g, m0, n0;
        tile_of(prm, tm, t, g, m0, n0);
        const int nk = (prm.p[g].K + BK - 1) / BK;
        // the first tile's weight stages go out before the programmatic wait
        int pre = 0;
        if (!waited) {
          pre = min(PSTAGES, nk);
          for (int i = 0; i < pre; ++i) {
            mbar_expect_tx(&full[i], A_BYTES + B_BYTES);
            tma_load_2d(sB + i * B_BYTES, &prm.tb[g], &full[i], i * BK, n0);
          }
          grid_dep_wait();
          grid_dep_trigger();
          waited = true;
          for (int i = 0; i < pre; ++i) tma_load_2d(sA + i * A_BYTES, &prm.ta[g], &full[i], i * BK, m0);
          it = pre;
        }
        for (int kb = pre; kb < nk; ++kb, ++it) {
          const int s = it % PSTAGES;
          const uint32_t r = it / PSTAGES;
          if (r > 0 && !mbar_wait(&empty[s], (r & 1) ^ 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], A_BYTES + B_BYTES);
          tma_load_2d(sA + s * A_BYTES, &prm.ta[g], &full[s], kb * BK, m0);
          tma_load_2d(sB + s * B_BYTES, &prm.tb[g], &full[s], kb * BK, n0);
        }
      }
      if (!waited) {
        grid_dep_wait();
        grid_dep_trigger();
      }
      // drain: never leave the CTA while copies may still land in shared memory
      for (int i = max(0, it - PSTAGES); i < it; ++i) mbar_wait(&full[i % PSTAGES], (i / PSTAGES) & 1);
    } else {
      grid_dep_wait();
      grid_dep_trigger();
    }
  } else if (warp == 1) {
    grid_dep_wait();
    grid_dep_trigger();
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = instr_desc<PBN>();
      int it = 0, j = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++j) {
        int g, m0, n0;
        tile_of(prm, tm, t, g, m0, n0);
        const int nk = (prm.p[g].K + BK - 1) / BK;
        const int b = j & 1;
        const uint32_t u = (uint32_t)(j >> 1);
        // accumulator b must have been drained by the epilogue of its previous tile
        if (u > 0 && !mbar_wait(&tempty[b], (u & 1) ^ 1)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + (uint32_t)(b * PBN);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % PSTAGES;
          if (!mbar_wait(&full[s], (it / PSTAGES) & 1)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint64_t ad = smem_desc_sw128(sA + s * A_BYTES);
          const uint64_t bd = smem_desc_sw128(sB + s * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_f16(d, ad + (uint64_t)(2 * kk), bd + (uint64_t)(2 * kk), idesc,
                     (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&tfull[b]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5), overlapped with the next tile's MMAs ----------------
    grid_dep_wait();
    grid_dep_trigger();
    const int quad = warp & 3;
    int j = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++j) {
      const int b = j & 1;
      const bool ok = mbar_wait(&tfull[b], (uint32_t)(j >> 1) & 1);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (!__all_sync(0xffffffffu, ok)) break;
      int g, m0, n0;
      tile_of(prm, tm, t, g, m0, n0);
      const TcProblem& P = prm.p[g];
      persist_epilogue<EPI>(P, g, m0 + quad * 32 + lane, n0,
                            tmem + (uint32_t)(b * PBN) + ((uint32_t)(quad * 32) << 16));
      // accumulator b is free again
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_plain(&tempty[b]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * PBN));
  }
}

// ---------------------------------------------------------------------------
// Two-SM variant of the persistent kernel (tcgen05 cta_group::2). A cluster of two
// CTAs (a CTA pair on neighbouring SMs) owns 256 x 256 output tiles: each CTA TMA-loads
// its own 128 rows of A and its own 128 rows (output columns) of B from this GPU's
// memory -- no multicast -- so a pair moves 2 x 32 KB per K-block for an M=256 x N=256 x
// K=64 product, against 48 KB per SM for the one-SM 128 x 256 tile. The even CTA (the
// leader) issues tcgen05.mma.cta_group::2 (M = 256, N = 256) reading both CTAs' shared
// memory; each CTA's TMEM receives its 128 rows of the accumulator, which its own four
// epilogue warps drain. Synchronisation:
//   full[s]   (leader)  both CTAs' copies complete_tx on it (mbarrier address with the
//                       peer bit cleared); the leader's producer arms it for 64 KB
//   empty[s]  (each)    the leader's commit multicast to both CTAs: stage s is free
//   tfull[b]  (each)    the leader's commit multicast: accumulator b holds a tile
//   tempty[b] (leader)  8 arrivals, the four epilogue warps of each CTA: b is drained
constexpr int QBM = 256, QSTAGES = 6;
constexpr uint32_t PEER_MASK = 0xFEFFFFFFu;  // shared::cluster address -> the even CTA's

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                 int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(saddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(saddr(bar) & PEER_MASK), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z),
      "r"(z), "r"(z), "r"(z), "r"(z), "r"(z));
}
// Arrive on barrier `bar` of both CTAs of the pair when the leader's MMAs so far complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
      ::"r"(saddr(bar)), "h"((unsigned short)3)
      : "memory");
}
// Arrive on the leader's copy of barrier `bar` (the same shared-memory offset).
__device__ __forceinline__ void mbar_arrive_leader(uint64_t* bar) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(remote) : "r"(saddr(bar)));
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

template <int EPI>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_gemm_tc_pair(const __grid_constant__ TcParams prm, const __grid_constant__ TileMap tm) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = BM * BK * 2, B_BYTES = (PBN / 2) * BK * 2;
  unsigned char* sA = base;
  unsigned char* sB = base + QSTAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + QSTAGES * B_BYTES);
  uint64_t* empty = full + QSTAGES;
  uint64_t* tfull = empty + QSTAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  const int total = tm.base[prm.n_problems];
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < QSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     saddr(tmem_slot)),
                 "r"(2 * PBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers initialised before any remote arrival
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      int it = 0;
      bool ok = true, waited = false;
      for (int t = pair; t < total && ok; t += npairs) {
        int g, m0, n0;
        tile_of(prm, tm, t, g, m0, n0);
        m0 = m0 * (QBM / BM);  // tile_of counts rows in BM units; pair tiles are QBM rows
        const int am = m0 + (int)rank * BM, bn = n0 + (int)rank * (PBN / 2);
        const int nk = (prm.p[g].K + BK - 1) / BK;
        int pre = 0;
        if (!waited) {  // the first tile's weight stages go out before the programmatic wait
          pre = min(QSTAGES, nk);
          for (int i = 0; i < pre; ++i) {
            if (leader) mbar_expect_tx(&full[i], 2 * (A_BYTES + B_BYTES));
            tma_load_2d_pair(sB + i * B_BYTES, &prm.tb[g], &full[i], i * BK, bn);
          }
          grid_dep_wait();
          grid_dep_trigger();
          waited = true;
          for (int i = 0; i < pre; ++i)
            tma_load_2d_pair(sA + i * A_BYTES, &prm.ta[g], &full[i], i * BK, am);
          it = pre;
        }
        for (int kb = pre; kb < nk; ++kb, ++it) {
          const int s = it % QSTAGES;
          const uint32_t r = it / QSTAGES;
          if (r > 0 && !mbar_wait(&empty[s], (r & 1) ^ 1)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(&full[s], 2 * (A_BYTES + B_BYTES));
          tma_load_2d_pair(sA + s * A_BYTES, &prm.ta[g], &full[s], kb * BK, am);
          tma_load_2d_pair(sB + s * B_BYTES, &prm.tb[g], &full[s], kb * BK, bn);
        }
      }
      if (!waited) {
        grid_dep_wait();
        grid_dep_trigger();
      }
      // drain: the last stages are free again once the leader's MMAs have read them
      for (int i = max(0, it - QSTAGES); i < it; ++i) {
        const uint32_t r = i / QSTAGES;
        mbar_wait(&empty[i % QSTAGES], r & 1);
      }
    } else {
      grid_dep_wait();
      grid_dep_trigger();
    }
  } else if (warp == 1) {
    grid_dep_wait();
    grid_dep_trigger();
    if (leader && lane == 0) {
      // ---------------- MMA issuer (leader only) ----------------
      const uint32_t idesc = (1u << 4) | ((uint32_t)(PBN >> 3) << 17) | ((uint32_t)(QBM >> 4) << 24);
      int it = 0, j = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += npairs, ++j) {
        int g, m0, n0;
        tile_of(prm, tm, t, g, m0, n0);
        const int nk = (prm.p[g].K + BK - 1) / BK;
        const int b = j & 1;
        const uint32_t u = (uint32_t)(j >> 1);
        if (u > 0 && !mbar_wait(&tempty[b], (u & 1) ^ 1)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + (uint32_t)(b * PBN);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % QSTAGES;
          if (!mbar_wait(&full[s], (it / QSTAGES) & 1)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint64_t ad = smem_desc_sw128(sA + s * A_BYTES);
          const uint64_t bd = smem_desc_sw128(sB + s * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_f16_pair(d, ad + (uint64_t)(2 * kk), bd + (uint64_t)(2 * kk), idesc,
                          (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit_pair(&empty[s]);
        }
        if (ok) umma_commit_pair(&tfull[b]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
    grid_dep_wait();
    grid_dep_trigger();
    const int quad = warp & 3;
    int j = 0;
    for (int t = pair; t < total; t += npairs, ++j) {
      const int b = j & 1;
      const bool ok = mbar_wait(&tfull[b], (uint32_t)(j >> 1) & 1);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (!__all_sync(0xffffffffu, ok)) break;
      int g, m0, n0;
      tile_of(prm, tm, t, g, m0, n0);
      m0 = m0 * (QBM / BM) + (int)rank * BM;
      persist_epilogue<EPI>(prm.p[g], g, m0 + quad * 32 + lane, n0,
                            tmem + (uint32_t)(b * PBN) + ((uint32_t)(quad * 32) << 16));
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_leader(&tempty[b]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the pair's MMAs may still use its memory
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * PBN));
  }
}

constexpr int pair_smem_bytes() {
  return 1024 + QSTAGES * (BM * BK * 2 + (PBN / 2) * BK * 2) + (2 * QSTAGES + 4) * 8 + 16;
}

// Launch of the pair kernel: clusters of two CTAs, as many pairs as can be resident
// (cudaOccupancyMaxActiveClusters), each walking 256 x 256 tiles.
template <int EPI>
int launch_tc_pair(const TcParams& prm, const TileMap& tm, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  static bool done[64] = {};
  static int max_clusters[64] = {};
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = pair_smem_bytes();
  cfg.stream = st;
  cfg.attrs = attr;
  if (dev < 64 && !done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_tc_pair<EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         pair_smem_bytes());
    int n = 0;
    if (e == cudaSuccess) {
      cfg.gridDim = dim3(148);
      cfg.numAttrs = 1;
      e = cudaOccupancyMaxActiveClusters(&n, k_gemm_tc_pair<EPI>, &cfg);
    }
    if (e != cudaSuccess || n < 1) {
      rwkv_set_error("gemm_tc_pair: setup: %s (%d clusters)", cudaGetErrorString(e), n);
      return RWKV_ERR_CUDA;
    }
    max_clusters[dev] = n;
    done[dev] = true;
  }
  const int total = tm.base[prm.n_problems];
  const int pairs = min(total, dev < 64 ? max_clusters[dev] : 70);
  cfg.gridDim = dim3(2 * pairs);
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.numAttrs = rwkv_chain_take_pdl() ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemm_tc_pair<EPI>, prm, tm);
  if (e != cudaSuccess) {
    rwkv_set_error("gemm_tc_pair: launch failed: %s", cudaGetErrorString(e));
    return RWKV_ERR_CUDA;
  }
  return rwkv_check_launch("gemm_tc_pair");
}

constexpr int persist_smem_bytes() {
  return 1024 + PSTAGES * (BM * BK * 2 + PBN * BK * 2) + (2 * PSTAGES + 4) * 8 + 16;
}

template <int EPI>
int launch_tc_persist(const TcParams& prm, const TileMap& tm, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  static bool done[64] = {};
  static int n_sm[64] = {};
  if (dev < 64 && !done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_tc_persist<EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         persist_smem_bytes());
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
      rwkv_set_error("gemm_tc_persist: setup: %s", cudaGetErrorString(e));
      return RWKV_ERR_CUDA;
    }
    done[dev] = true;
  }
  const int total = tm.base[prm.n_problems];
  const int grid = min(total, dev < 64 ? n_sm[dev] : 148);
  return rwkv_launch("gemm_tc_persist", k_gemm_tc_persist<EPI>, dim3(grid), dim3(NTHREADS),
                     (size_t)persist_smem_bytes(), st, prm, tm);
}

}  // namespace

// True when every problem fits the tcgen05 path (K multiple of 64, aligned operands).
template <int BN, int STAGES>
int gemm_tc_launch_cfg(const rwkv7_gemm_problem* p, int n, int epi, int splits, float* ws,
                       bool defer, cudaStream_t st);

// RWKV_B200_GEMM_PERSIST=0 turns the persistent large-problem kernel off.
bool gemm_persist_enabled() {
  static const bool on = [] {
    const char* e = getenv("RWKV_B200_GEMM_PERSIST");
    return !(e && e[0] == '0');
  }();
  return on;
}

// SM count of the current device (cached per device).
static int device_sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// RWKV_B200_GEMM_PAIR=0 keeps large problems on the one-SM persistent kernel.
bool gemm_pair_enabled() {
  static const bool on = [] {
    const char* e = getenv("RWKV_B200_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Persistent tiles over every problem of the group (splits = 1): 256 x 256 on CTA pairs
// (cta_group::2), or 128 x 256 on single CTAs.
int gemm_tc_launch_persist(const rwkv7_gemm_problem* p, int n, int epi, cudaStream_t st) {
  // CTA pairs when they all get a tile (>= one 256 x 256 tile per pair); a group of fewer
  // tiles (e.g. the prefill FFN value, 64 tiles) runs faster on the single-CTA kernel,
  // whose 128-row tiles reach more SMs
  int pair_tiles = 0;
  for (int i = 0; i < n; ++i) pair_tiles += ((p[i].M + QBM - 1) / QBM) * ((p[i].N + PBN - 1) / PBN);
  const bool pair = gemm_pair_enabled() && pair_tiles >= device_sm_count() / 2;
  const int tile_m = pair ? QBM : BM, box_n = pair ? PBN / 2 : PBN;
  TcParams prm;
  TileMap tm;
  memset(&prm, 0, sizeof(prm));
  memset(&tm, 0, sizeof(tm));
  prm.n_problems = n;
  prm.splits = 1;
  for (int i = 0; i < n; ++i) {
    int rc = make_map(&prm.ta[i], p[i].A, p[i].M, p[i].K, p[i].lda, BM);
    if (rc) return rc;
    rc = make_map(&prm.tb[i], p[i].B, p[i].N, p[i].K, p[i].ldb, box_n);
    if (rc) return rc;
    prm.p[i].C = p[i].C;
    prm.p[i].R = p[i].R;
    prm.p[i].M = p[i].M;
    prm.p[i].N = p[i].N;
    prm.p[i].K = p[i].K;
    prm.p[i].ldc = p[i].ldc;
    tm.tiles_m[i] = (p[i].M + tile_m - 1) / tile_m;
    tm.base[i + 1] = tm.base[i] + tm.tiles_m[i] * ((p[i].N + PBN - 1) / PBN);
  }
  if (pair) switch (epi) {
    case RWKV_EPI_STORE: return launch_tc_pair<RWKV_EPI_STORE>(prm, tm, st);
    case RWKV_EPI_RESID: return launch_tc_pair<RWKV_EPI_RESID>(prm, tm, st);
    case RWKV_EPI_RELUSQ: return launch_tc_pair<RWKV_EPI_RELUSQ>(prm, tm, st);
    case RWKV_EPI_STORE_F32: return launch_tc_pair<RWKV_EPI_STORE_F32>(prm, tm, st);
    case EPI_ARGMAX: return launch_tc_pair<EPI_ARGMAX>(prm, tm, st);
  }
  switch (epi) {
    case RWKV_EPI_STORE: return launch_tc_persist<RWKV_EPI_STORE>(prm, tm, st);
    case RWKV_EPI_RESID: return launch_tc_persist<RWKV_EPI_RESID>(prm, tm, st);
    case RWKV_EPI_RELUSQ: return launch_tc_persist<RWKV_EPI_RELUSQ>(prm, tm, st);
    case RWKV_EPI_STORE_F32: return launch_tc_persist<RWKV_EPI_STORE_F32>(prm, tm, st);
    case EPI_ARGMAX: return launch_tc_persist<EPI_ARGMAX>(prm, tm, st);
  }
  rwkv_set_error("gemm_tc_persist: epilogue %d not supported", epi);
  return RWKV_ERR_ARG;
}

// Tile configuration and split-K by problem size. Large grids: 128 x 128 tiles,
// 3 stages (two CTAs per SM). Small grids (batched decode): 128 x 64 tiles with 6
// stages (144 KiB of operands in flight per CTA) and, when still fewer than 48
// tiles, a K split with at least 4 K-blocks per slice and at most one wave of CTAs. `ws` takes the split-K fp32
// partial tiles (ws_floats floats; no initial value needed). With `splits_out`
// non-null the split-K reduce is left to the consumer: *splits_out receives the
// number of K-slices parked in ws ([splits][M][N] fp32 per problem, problems back to
// back), 1 when the GEMM wrote its output directly.

int gemm_tc_launch(const rwkv7_gemm_problem* p, int n, int epi, float* ws, size_t ws_floats,
                   cudaStream_t st, int* splits_out) {
  int tiles128 = 0, tiles64 = 0, min_kb = 1 << 30;
  size_t mn = 0;
  bool n4 = true;
  for (int i = 0; i < n; ++i) {
    tiles128 += ((p[i].M + BM - 1) / BM) * ((p[i].N + 127) / 128);
    tiles64 += ((p[i].M + BM - 1) / BM) * ((p[i].N + 63) / 64);
    min_kb = min(min_kb, (p[i].K + BK - 1) / BK);
    mn += (size_t)p[i].M * p[i].N;
    n4 = n4 && p[i].N % 4 == 0 && p[i].ldc % 2 == 0;
  }
  if (splits_out) *splits_out = 1;
  if (tiles128 >= 148) {
    bool wide = epi != RWKV_EPI_LORA_ACT && epi != RWKV_EPI_LORA_ACT2;
    for (int i = 0; i < n; ++i) wide = wide && p[i].N >= PBN;
    if (wide && gemm_persist_enabled()) return gemm_tc_launch_persist(p, n, epi, st);
    return gemm_tc_launch_cfg<128, 3>(p, n, epi, 1, ws, false, st);
  }
  int splits = 1;
  if (ws && n4 && tiles64 < 48 && epi != EPI_ARGMAX) {
    // as many K-slices (of at least 4 K-blocks) as keep the grid within one wave of
    // one CTA per SM: a second wave costs more than the slices save
    splits = max(1, min(min_kb / 4, device_sm_count() / tiles64));
    while (splits > 1 && (size_t)splits * mn > ws_floats) --splits;
  }
  if (splits_out) *splits_out = splits;
  // more 128 x 64 tiles than SMs (the prefill LoRA-down): 3 stages (72 KiB) let two or
  // three CTAs share an SM, so the grid runs as one wave instead of two
  if (splits == 1 && tiles64 > device_sm_count())
    return gemm_tc_launch_cfg<64, 3>(p, n, epi, 1, ws, false, st);
  return gemm_tc_launch_cfg<64, 6>(p, n, epi, splits, ws, splits_out != nullptr, st);
}

template <int BN, int STAGES>
int gemm_tc_launch_cfg(const rwkv7_gemm_problem* p, int n, int epi, int splits, float* ws,
                       bool defer, cudaStream_t st) {
  TcParams prm;
  memset(&prm, 0, sizeof(prm));
  prm.n_problems = n;
  prm.splits = splits;
  int gx = 0, gy = 0;
  size_t ws_off = 0, total = 0;
  for (int i = 0; i < n; ++i) total += (size_t)p[i].M * p[i].N;
  for (int i = 0; i < n; ++i) {
    int rc = make_map(&prm.ta[i], p[i].A, p[i].M, p[i].K, p[i].lda, BM);
    if (rc) return rc;
    rc = make_map(&prm.tb[i], p[i].B, p[i].N, p[i].K, p[i].ldb, BN);
    if (rc) return rc;
    prm.p[i].C = p[i].C;
    prm.p[i].R = p[i].R;
    prm.p[i].M = p[i].M;
    prm.p[i].N = p[i].N;
    prm.p[i].K = p[i].K;
    prm.p[i].ldc = p[i].ldc;
    prm.p[i].ws = splits > 1 ? ws + ws_off * splits : nullptr;
    ws_off += (size_t)p[i].M * p[i].N;
    gx = max(gx, (p[i].N + BN - 1) / BN);
    gy = max(gy, (p[i].M + BM - 1) / BM);
  }
  (void)total;
  dim3 grid(gx, gy, n * splits);
  int rc;
  switch (epi) {
    case RWKV_EPI_STORE: rc = launch_tc<BN, RWKV_EPI_STORE, STAGES>(prm, grid, st); break;
    case RWKV_EPI_RESID: rc = launch_tc<BN, RWKV_EPI_RESID, STAGES>(prm, grid, st); break;
    case RWKV_EPI_RELUSQ: rc = launch_tc<BN, RWKV_EPI_RELUSQ, STAGES>(prm, grid, st); break;
    case RWKV_EPI_STORE_F32: rc = launch_tc<BN, RWKV_EPI_STORE_F32, STAGES>(prm, grid, st); break;
    case RWKV_EPI_LORA_ACT: rc = launch_tc<BN, RWKV_EPI_LORA_ACT, STAGES>(prm, grid, st); break;
    case EPI_ARGMAX: rc = launch_tc<BN, EPI_ARGMAX, STAGES>(prm, grid, st); break;
    default: rc = launch_tc<BN, RWKV_EPI_LORA_ACT2, STAGES>(prm, grid, st); break;
  }
  if (rc || splits == 1 || defer) return rc;
  ReduceParams rp;
  rp.n_problems = n;
  rp.splits = splits;
  size_t max_mn = 0;
  for (int i = 0; i < n; ++i) {
    rp.p[i] = prm.p[i];
    max_mn = max(max_mn, (size_t)p[i].M * p[i].N);
  }
  dim3 rgrid((unsigned)((max_mn / 4 + 255) / 256), n);
  auto red = epi == RWKV_EPI_STORE     ? k_splitk_reduce<RWKV_EPI_STORE>
             : epi == RWKV_EPI_RESID     ? k_splitk_reduce<RWKV_EPI_RESID>
             : epi == RWKV_EPI_RELUSQ    ? k_splitk_reduce<RWKV_EPI_RELUSQ>
             : epi == RWKV_EPI_STORE_F32 ? k_splitk_reduce<RWKV_EPI_STORE_F32>
             : epi == RWKV_EPI_LORA_ACT  ? k_splitk_reduce<RWKV_EPI_LORA_ACT>
                                         : k_splitk_reduce<RWKV_EPI_LORA_ACT2>;
  return rwkv_launch("splitk_reduce", red, rgrid, dim3(256), 0, st, rp);
}

// Self-test of the pipeline's bounded wait: one thread waits on an mbarrier that
// nothing ever arrives on, through the same mbar_wait the GEMM kernels use. The wait
// must give up, set the device error flag and let the kernel return.
namespace {
__global__ void k_wait_selftest_tc(int* out) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    out[0] = mbar_wait(&bar, 0) ? 0 : 1;
  }
}
}  // namespace
int wait_selftest_tc(int* out, cudaStream_t st) {
  return rwkv_launch("wait_selftest_tc", k_wait_selftest_tc, dim3(1), dim3(32), 0, st, out);
}

// Host read of the device timeout flag (cleared on read); nonzero means a bounded wait gave up.
int gemm_tc_timeout_flag() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_tc_timeout, sizeof(int));
  if (v) {
    int z = 0;
    cudaMemcpyToSymbol(g_tc_timeout, &z, sizeof(int));
  }
  return v;
}

// ---- public GEMM entry ------------------------------------------------------
// Validation of a group of up to 4 problems (shapes, strides, alignment).
int gemm_validate(const rwkv7_gemm_problem* p, int n) {
  if (!p || n < 1 || n > 4) {
    rwkv_set_error("rwkv7_gemm_f16: need 1..4 problems (got %d)", n);
    return RWKV_ERR_ARG;
  }
  for (int i = 0; i < n; ++i) {
    const rwkv7_gemm_problem& q = p[i];
    if (q.M < 0 || q.N < 0 || q.K <= 0 || q.K % 32 || q.N % 2 || q.lda % 8 || q.ldb % 8 ||
        q.ldc % 2 || !q.A || !q.B || !q.C || (reinterpret_cast<uintptr_t>(q.C) & 7) ||
        (reinterpret_cast<uintptr_t>(q.R) & 7) || q.lda < q.K || q.ldb < q.K || q.ldc < q.N) {
      rwkv_set_error("rwkv7_gemm_f16: bad problem %d (M=%d N=%d K=%d lda=%d ldb=%d ldc=%d)", i,
                     q.M, q.N, q.K, q.lda, q.ldb, q.ldc);
      return RWKV_ERR_ARG;
    }
    if ((reinterpret_cast<uintptr_t>(q.A) | reinterpret_cast<uintptr_t>(q.B)) & 15) {
      rwkv_set_error("rwkv7_gemm_f16: A and B must be 16-byte aligned (problem %d)", i);
      return RWKV_ERR_ARG;
    }
  }
  return RWKV_OK;
}

// Every GEMM runs on the tcgen05 kernels (K % 64 == 32 included: the last K-block's
// tensor-map box reaches past K and the TMA fills it with zeros). `ws` is the split-K
// scratch; with `splits_out` non-null a split-K GEMM leaves its fp32 K-slices in ws for
// the consumer to sum (*splits_out > 1) instead of launching the reduce.
int gemm_launch_ws(const rwkv7_gemm_problem* problems, int n, int epi, float* ws,
                   size_t ws_floats, cudaStream_t st, int* splits_out) {
  return gemm_tc_launch(problems, n, epi, ws, ws_floats, st, splits_out);
}

extern "C" int rwkv7_gemm_f16(const rwkv7_gemm_problem* problems, int n_problems, int epilogue,
                              void* stream) {
  rwkv_chain_begin();
  int rc = gemm_validate(problems, n_problems);
  if (rc) return rc;
  if (epilogue < RWKV_EPI_STORE || epilogue > RWKV_EPI_LORA_ACT2) {
    rwkv_set_error("rwkv7_gemm_f16: unknown epilogue %d", epilogue);
    return RWKV_ERR_ARG;
  }
  for (int i = 0; i < n_problems; ++i)
    if (epilogue == RWKV_EPI_RESID && !problems[i].R) {
      rwkv_set_error("rwkv7_gemm_f16: residual epilogue needs R (problem %d)", i);
      return RWKV_ERR_ARG;
    }
  return gemm_launch_ws(problems, n_problems, epilogue, nullptr, 0, (cudaStream_t)stream, nullptr);
}
