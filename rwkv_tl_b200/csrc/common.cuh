// Shared device helpers for the RWKV-7 sm_100a kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/rwkv_b200.h"

#define RWKV_HD 64  // head size N, fixed for RWKV-7
#define RWKV_RANK_V 32
#define RWKV_RANK_W 64
#define RWKV_RANK_A 64
#define RWKV_RANK_G 128
#define RWKV_RANK_SUM 288  // v | w | a | g packed order

// Rounding semantics of the two reference paths (see include/rwkv_b200.h).
enum { SEM_DECODE = 0, SEM_PREFILL = 1 };

__device__ __forceinline__ float r16(float x) { return __half2float(__float2half_rn(x)); }
__device__ __forceinline__ float h2f(__half x) { return __half2float(x); }
__device__ __forceinline__ __half f2h(float x) { return __float2half_rn(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// warp_sum for a layout in which one lane does the work of P lanes: lane j holds the
// P partials of "lanes" P * j .. P * j + P - 1, and a group of 32 / P lanes stands for
// one warp. Replays warp_sum's butterfly (offsets >= P as shuffles by offset / P,
// smaller ones as adds within the lane), so the result rounds exactly like warp_sum
// over the 32 original partials. P = 1 is warp_sum itself.
template <int P>
__device__ __forceinline__ float warp_sum_p(float (&p)[P]) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    if (off >= P) {
#pragma unroll
      for (int q = 0; q < P; ++q) p[q] += __shfl_xor_sync(0xffffffffu, p[q], off / P);
    } else {
      float t[P];
#pragma unroll
      for (int q = 0; q < P; ++q) t[q] = p[q] + p[q ^ off];
#pragma unroll
      for (int q = 0; q < P; ++q) p[q] = t[q];
    }
  }
  return p[0];
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// 4 x fp16 <-> float4 through one 8-byte access.
__device__ __forceinline__ float4 load_h4(const __half* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __half2 a = *reinterpret_cast<__half2*>(&u.x), b = *reinterpret_cast<__half2*>(&u.y);
  float2 fa = __half22float2(a), fb = __half22float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}
__device__ __forceinline__ void store_h4(__half* p, float4 v) {
  __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

// GEMM epilogue for one output pair (c0, c1) at element offset o of C; `prob` is the
// index of the problem in a grouped launch (RWKV_EPI_LORA_ACT: 1 -> tanh, 3 -> sigmoid).
template <int EPI>
__device__ __forceinline__ void epi_store2(void* C, size_t o, float c0, float c1,
                                           const __half* R, int prob) {
  if (EPI == RWKV_EPI_STORE_F32) {
    *reinterpret_cast<float2*>(static_cast<float*>(C) + o) = make_float2(c0, c1);
    return;
  }
  __half2 h;
  if (EPI == RWKV_EPI_STORE) {
    h = __floats2half2_rn(c0, c1);
  } else if (EPI == RWKV_EPI_RESID) {
    const float2 r = __half22float2(*reinterpret_cast<const __half2*>(R + o));
    h = __floats2half2_rn(r.x + r16(c0), r.y + r16(c1));
  } else if (EPI == RWKV_EPI_RELUSQ) {
    const float h0 = fmaxf(r16(c0), 0.f), h1 = fmaxf(r16(c1), 0.f);
    h = __floats2half2_rn(h0 * h0, h1 * h1);
  } else {  // RWKV_EPI_LORA_ACT / RWKV_EPI_LORA_ACT2
    float a = r16(c0), b = r16(c1);
    if (prob == 1) {
      a = tanhf(a);
      b = tanhf(b);
    } else if (prob == 3) {
      a = 1.0f / (1.0f + expf(-a));
      b = 1.0f / (1.0f + expf(-b));
    }
    h = __floats2half2_rn(a, b);
    if (EPI == RWKV_EPI_LORA_ACT2 && (prob == 1 || prob == 3)) {
      // fp32 activation kept as fp16 hi + lo: lo goes `lo_off` columns to the right
      const int lo_off = prob == 1 ? 64 : 128;
      const float2 hf = __half22float2(h);
      *reinterpret_cast<__half2*>(static_cast<__half*>(C) + o + lo_off) =
          __floats2half2_rn(a - hf.x, b - hf.y);
    }
  }
  *reinterpret_cast<__half2*>(static_cast<__half*>(C) + o) = h;
}

// Block-wide sum of NV floats; `red` needs 32*NV floats of shared memory.
template <int NV>
__device__ __forceinline__ void block_sum(float (&v)[NV], float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] = warp_sum(v[i]);
  __syncthreads();
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < NV; ++i) red[wid * NV + i] = v[i];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float s = 0.f;
    for (int w = 0; w < nw; ++w) s += red[w * NV + i];
    v[i] = s;
  }
  __syncthreads();
}

// Host side: record an error message for rwkv_b200_last_error().
void rwkv_set_error(const char* fmt, ...);
int rwkv_check_launch(const char* what);

// Programmatic dependent launch. Kernels of a library call after its first are
// launched with programmatic stream serialization. Every such kernel calls
// grid_dep_wait() before its first access to memory written by an earlier kernel
// (it returns once the preceding grid has completed and its writes are visible) and
// only then grid_dep_trigger(), which lets the next kernel launch and run its
// prologue (barrier and TMEM set-up, the GEMM's first weight tiles) while this one
// works. Triggering after the wait keeps the chain one kernel deep: a kernel is never
// launched before its predecessor's predecessor has completed, so data written two
// or more kernels back is complete and visible to it.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
#define RWKV_GRID_DEP_ENTRY() \
  do {                        \
    grid_dep_wait();          \
    grid_dep_trigger();       \
  } while (0)

// Internal GEMM epilogue of the lm head's greedy path: C is a uint64 [M] array of
// per-row keys (ordered fp16 logit << 32 | ~column), combined with atomicMax.
constexpr int EPI_ARGMAX = 6;

// Monotonic 64-bit key of (fp16-rounded value, column): a larger key is a larger
// value, and among equal values the smaller column (torch.argmax picks the first).
__device__ __forceinline__ unsigned long long argmax_key(float v, int col) {
  uint32_t u = __float_as_uint(v == 0.f ? 0.f : v);  // -0 and +0 compare equal
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (0xFFFFFFFFu - (uint32_t)col);
}

// A residual sum res + A @ B whose split-K GEMM left its `splits` fp32 K-slices in
// ws ([splits][M][C]) for the consuming row kernel to finish; ws == nullptr: none.
struct PendingResid {
  const float* ws;
  const __half* res;
  int splits;
};

// Large token batches (M >= 1024) run the row, gate and GroupNorm kernels with 8
// channels per thread; RWKV_B200_NARROW=1 keeps the narrow layouts at every size
// (their sums replay the same summation trees, so results are bit-identical).
bool rwkv_rows_wide(int M, int C);
bool rwkv_pdl_enabled();  // RWKV_B200_PDL=0 turns the attribute off (plain stream order)
// Start of a library call: its first launch depends on whatever the caller queued
// before (copies, memsets, other libraries' kernels) in plain stream order; only
// launches after it, within the call, get the programmatic edge.
void rwkv_chain_begin();
bool rwkv_chain_take_pdl();  // attribute for this launch? (false once per chain begin)

template <typename... KArgs, typename... Args>
int rwkv_launch(const char* name, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = rwkv_chain_take_pdl() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
  if (e != cudaSuccess) {
    rwkv_set_error("%s: launch failed: %s", name, cudaGetErrorString(e));
    return RWKV_ERR_CUDA;
  }
  return rwkv_check_launch(name);
}
