// Building blocks shared by the small-batch decode paths (decode_gemv.cu and
// decode_persist.cu): layer weight pointers, warp GEMV over 16-byte weight chunks,
// register LayerNorm, multi-value warp reductions and async-copy helpers.
#pragma once

#include "common.cuh"

namespace dec {

// Order-independent accumulation across CTAs. Each partial sum is rounded once to a
// 64-bit fixed-point integer with 32 fraction bits and added with an integer atomic.
// Integer addition is associative, so the total -- and everything computed from it --
// is the same bits whatever order the CTAs' additions land in (float atomics are not).
// Range |partial| < 2^31 (activations are fp16, < 65504); resolution 2^-32, far below
// the fp16 rounding that every sum receives.
__device__ __forceinline__ void fx_add(long long* p, float v) {
  atomicAdd(reinterpret_cast<unsigned long long*>(p),
            static_cast<unsigned long long>(__float2ll_rn(v * 4294967296.0f)));
}
__device__ __forceinline__ float fx_val(long long x) {
  return static_cast<float>(x) * 2.3283064365386963e-10f;  // 2^-32
}

constexpr int MAXB = 8;
constexpr int NT = 256;

struct DecLayer {
  const __half *ln1_w, *ln1_b, *ln2_w, *ln2_b, *mix6, *w_rkv, *w_lora_dn, *w_lora_up;
  const __half *w0, *a0, *v0, *k_k, *k_a, *r_k, *lnx_w, *lnx_b, *w_o, *ffn_x_k, *w_fk, *w_fv;
};

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void l2_prefetch_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(src));
}

__device__ __forceinline__ float dot8(uint4 w, uint4 x) {
  const __half2* a = reinterpret_cast<const __half2*>(&w);
  const __half2* b = reinterpret_cast<const __half2*>(&x);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 fa = __half22float2(a[i]), fb = __half22float2(b[i]);
    s += fa.x * fb.x;
    s += fa.y * fb.y;
  }
  return s;
}

// GEMV building blocks, one warp: gemv_load issues all RPW * CPL 16-byte loads of
// up to RPW weight rows (CPL = C / 256 chunks per lane per row) -- callable before
// griddepcontrol.wait -- and gemv_dot forms acc[r][b] against NB activation rows.
template <int CPL, int RPW>
__device__ __forceinline__ void gemv_load(const __half* const (&wrow)[RPW], int nrows, int lane,
                                          uint4 (&w)[RPW][CPL]) {
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int q = 0; q < CPL; ++q)
      if (r < nrows) w[r][q] = __ldg(reinterpret_cast<const uint4*>(wrow[r]) + lane + 32 * q);
}

template <int NB, int CPL, int RPW>
__device__ __forceinline__ void gemv_dot(const uint4 (&w)[RPW][CPL], const __half* const (&xv)[RPW],
                                         int nrows, int C, int lane, float (&acc)[RPW][NB]) {
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[r][b] = 0.f;
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    if (r >= nrows) continue;
#pragma unroll
    for (int q = 0; q < CPL; ++q)
#pragma unroll
      for (int b = 0; b < NB; ++b)
        acc[r][b] += dot8(w[r][q], reinterpret_cast<const uint4*>(xv[r] + (size_t)b * C)[lane + 32 * q]);
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[r][b] = warp_sum(acc[r][b]);
}

// LayerNorm of NB register-resident rows (thread holds channels tid + NT k) with one
// block reduction of (sum, sum of squares); fp32 statistics, fp16 output
// (F.layer_norm on an fp16 tensor, weight.py:6-15).
template <int NB, int CPL>
__device__ __forceinline__ void ln_regs(float (&x)[NB][CPL], const float (&lw)[CPL],
                                        const float (&lb)[CPL], int C, float* red) {
  float s[2 * NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    s[b] = 0.f;
    s[NB + b] = 0.f;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      s[b] += x[b][k];
      s[NB + b] += x[b][k] * x[b][k];
    }
  }
  block_sum<2 * NB>(s, red);
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const float mean = s[b] / C;
    const float var = fmaxf(s[NB + b] / C - mean * mean, 0.f);
    const float rstd = rsqrtf(var + 1e-5f);
#pragma unroll
    for (int k = 0; k < CPL; ++k) x[b][k] = r16((x[b][k] - mean) * rstd * lw[k] + lb[k]);
  }
}

// Rows base, base + 8, ... (< r1) of kernel A's stacked [W_rkv ; W_lora_dn]: weight row
// pointers and the mix each multiplies (r, k, v -> mixes 0, 2, 3; LoRA v, w, a, g ->
// Sum 8 per-lane partials across the warp (9 shuffles); lane l ends with the total of
// index (l >> 2) & 7.
__device__ __forceinline__ float reduce8(float (&p)[8], int lane) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool up = lane & 16;
    const float send = up ? p[i] : p[i + 4];
    const float keep = up ? p[i + 4] : p[i];
    p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool up = lane & 8;
    const float send = up ? p[i] : p[i + 2];
    const float keep = up ? p[i + 2] : p[i];
    p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  {
    const bool up = lane & 4;
    const float send = up ? p[0] : p[1];
    const float keep = up ? p[1] : p[0];
    p[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  p[0] += __shfl_xor_sync(0xffffffffu, p[0], 2);
  return p[0] + __shfl_xor_sync(0xffffffffu, p[0], 1);
}

// ---------------------------------------------------------------------------

}  // namespace dec
