// Grouped fp16 GEMM with fused epilogues (warp-level mma.sync m16n8k16).
//
// C[M, N] = epi(A[M, K] @ B[N, K]^T), fp32 accumulation. This is the portable
// tensor-core path; the tcgen05 kernel in gemm_tc.cu replaces it for the large
// prefill / batched-decode problems. Tile 128x128x32, 4-stage cp.async
// pipeline, 8 warps (2 x 4, warp tile 64 x 32), XOR-swizzled shared memory
// read with ldmatrix.
#include <cstdlib>

#include "common.cuh"

namespace {

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 4, NTHREADS = 256;
constexpr int TILE_HALVES = BM * BK;  // per operand per stage (BM == BN)

struct GemmGroup {
  rwkv7_gemm_problem p[4];
  int n;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(sz));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// element offset of (row, 16B-chunk) inside a [rows][32] swizzled tile
__device__ __forceinline__ int swz(int row, int chunk) {
  return row * BK + ((chunk ^ ((row >> 1) & 3)) << 3);
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int EPI>
__global__ void __launch_bounds__(NTHREADS) k_gemm_mma(const GemmGroup grp) {
  RWKV_GRID_DEP_ENTRY();
  extern __shared__ __align__(128) __half smem[];
  if ((int)blockIdx.z >= grp.n) return;
  const rwkv7_gemm_problem& P = grp.p[blockIdx.z];
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  if (n0 >= P.N || m0 >= P.M) return;
  const __half* A = static_cast<const __half*>(P.A);
  const __half* B = static_cast<const __half*>(P.B);
  __half* sA = smem;
  __half* sB = smem + STAGES * TILE_HALVES;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp >> 2, wn = warp & 3;
  const int KT = P.K / BK;

  auto load_stage = [&](int stage, int kt) {
    const int k0 = kt * BK;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = tid + i * NTHREADS;  // 0..511
      const int row = idx >> 2, ch = idx & 3;
      const int gm = m0 + row, gn = n0 + row;
      const bool pa = gm < P.M, pb = gn < P.N;
      const __half* srcA = A + (size_t)(pa ? gm : 0) * P.lda + k0 + ch * 8;
      const __half* srcB = B + (size_t)(pb ? gn : 0) * P.ldb + k0 + ch * 8;
      cp_async16(smem_u32(sA + stage * TILE_HALVES + swz(row, ch)), srcA, pa);
      cp_async16(smem_u32(sB + stage * TILE_HALVES + swz(row, ch)), srcB, pb);
    }
  };

  float acc[4][4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[i][j][q] = 0.f;

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < KT) load_stage(s, s);
    cp_commit();
  }

  for (int kt = 0; kt < KT; ++kt) {
    cp_wait<STAGES - 2>();
    __syncthreads();
    const int nk = kt + STAGES - 1;
    if (nk < KT) load_stage(nk % STAGES, nk);
    cp_commit();
    const __half* tA = sA + (kt % STAGES) * TILE_HALVES;
    const __half* tB = sB + (kt % STAGES) * TILE_HALVES;
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t af[4][4];
#pragma unroll
      for (int mi = 0; mi < 4; ++mi) {
        const int row = wm * 64 + mi * 16 + (lane & 15);
        const int ch = kk * 2 + (lane >> 4);
        ldmatrix_x4(smem_u32(tA + swz(row, ch)), af[mi][0], af[mi][1], af[mi][2], af[mi][3]);
      }
      uint32_t bf[4][2];
#pragma unroll
      for (int nj = 0; nj < 2; ++nj) {
        const int row = wn * 32 + nj * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int ch = kk * 2 + ((lane >> 3) & 1);
        ldmatrix_x4(smem_u32(tB + swz(row, ch)), bf[2 * nj][0], bf[2 * nj][1], bf[2 * nj + 1][0],
                    bf[2 * nj + 1][1]);
      }
#pragma unroll
      for (int mi = 0; mi < 4; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) mma16816(acc[mi][ni], af[mi], bf[ni][0], bf[ni][1]);
    }
  }
  cp_wait<0>();

  const __half* R = static_cast<const __half*>(P.R);
#pragma unroll
  for (int mi = 0; mi < 4; ++mi) {
#pragma unroll
    for (int ni = 0; ni < 4; ++ni) {
      const int col = n0 + wn * 32 + ni * 8 + (lane & 3) * 2;
      if (col >= P.N) continue;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int row = m0 + wm * 64 + mi * 16 + (lane >> 2) + hh * 8;
        if (row >= P.M) continue;
        const size_t o = (size_t)row * P.ldc + col;
        epi_store2<EPI>(P.C, o, acc[mi][ni][2 * hh], acc[mi][ni][2 * hh + 1], R, blockIdx.z);
      }
    }
  }
}

template <int EPI>
int launch_group(const GemmGroup& g, cudaStream_t st) {
  const int smem = STAGES * TILE_HALVES * 2 * 2;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool done[64] = {};
  if (dev < 64 && !done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_mma<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      rwkv_set_error("gemm: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return RWKV_ERR_CUDA;
    }
    done[dev] = true;
  }
  int gx = 0, gy = 0;
  for (int i = 0; i < g.n; ++i) {
    gx = max(gx, (g.p[i].N + BN - 1) / BN);
    gy = max(gy, (g.p[i].M + BM - 1) / BM);
  }
  if (gx == 0 || gy == 0) return RWKV_OK;
  return rwkv_launch("gemm_mma", k_gemm_mma<EPI>, dim3(gx, gy, g.n), dim3(NTHREADS), smem, st, g);
}

}  // namespace

int gemm_validate(const rwkv7_gemm_problem* p, int n) {
  if (!p || n < 1 || n > 4) {
    rwkv_set_error("rwkv7_gemm_f16: need 1..4 problems (got %d)", n);
    return RWKV_ERR_ARG;
  }
  for (int i = 0; i < n; ++i) {
    const rwkv7_gemm_problem& q = p[i];
    if (q.M < 0 || q.N < 0 || q.K <= 0 || q.K % BK || q.N % 2 || q.lda % 8 || q.ldb % 8 ||
        q.ldc % 2 || !q.A || !q.B || !q.C || (reinterpret_cast<uintptr_t>(q.C) & 7) || q.lda < q.K || q.ldb < q.K || q.ldc < q.N) {
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

int gemm_mma_launch(const rwkv7_gemm_problem* problems, int n, int epi, cudaStream_t st) {
  GemmGroup g;
  g.n = n;
  for (int i = 0; i < n; ++i) g.p[i] = problems[i];
  switch (epi) {
    case RWKV_EPI_STORE: return launch_group<RWKV_EPI_STORE>(g, st);
    case RWKV_EPI_RESID: return launch_group<RWKV_EPI_RESID>(g, st);
    case RWKV_EPI_RELUSQ: return launch_group<RWKV_EPI_RELUSQ>(g, st);
    case RWKV_EPI_STORE_F32: return launch_group<RWKV_EPI_STORE_F32>(g, st);
    case RWKV_EPI_LORA_ACT: return launch_group<RWKV_EPI_LORA_ACT>(g, st);
    case RWKV_EPI_LORA_ACT2: return launch_group<RWKV_EPI_LORA_ACT2>(g, st);
  }
  rwkv_set_error("rwkv7_gemm_f16: unknown epilogue %d", epi);
  return RWKV_ERR_ARG;
}

bool gemm_tc_eligible(const rwkv7_gemm_problem* p, int n);
int gemm_tc_launch(const rwkv7_gemm_problem* p, int n, int epi, float* ws, size_t ws_floats,
                   cudaStream_t st, int* splits_out);

// Kernel choice by shape: the tcgen05 kernel when every problem has K % 64 == 0
// (all model projections; it picks its tile shape and split-K itself, `ws` being
// the split-K scratch), else the mma.sync kernel. RWKV_B200_GEMM=mma|tc forces one.
// With `splits_out` non-null a split-K GEMM leaves its fp32 K-slices in ws for the
// consumer to sum (*splits_out > 1) instead of launching the reduce.
int gemm_launch_ws(const rwkv7_gemm_problem* problems, int n, int epi, float* ws,
                   size_t ws_floats, cudaStream_t st, int* splits_out) {
  const char* e = getenv("RWKV_B200_GEMM");
  const bool force_mma = e && e[0] == 'm';
  if (force_mma || !gemm_tc_eligible(problems, n)) {
    if (splits_out) *splits_out = 1;
    return gemm_mma_launch(problems, n, epi, st);
  }
  return gemm_tc_launch(problems, n, epi, ws, ws_floats, st, splits_out);
}

int gemm_launch(const rwkv7_gemm_problem* problems, int n, int epi, cudaStream_t st) {
  return gemm_launch_ws(problems, n, epi, nullptr, 0, st, nullptr);
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
  return gemm_launch(problems, n_problems, epilogue, (cudaStream_t)stream);
}
