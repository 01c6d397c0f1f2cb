// Gate math + per-head L2 norm on the LoRA up-projection outputs.
//
// The up-projections themselves run as one grouped tcgen05 GEMM (gemm_tc.cu) over
// the padded rank buffer [M, 512] = v(32, zero-padded to 64) | tanh(w) hi, lo (64 + 64) | a(64) |
// sigmoid(g) hi, lo (128 + 128) and the K-major weights w_lora_up_t [C, 512], giving v12, w12, a12,
// g12 [M, C] (fp32 with decode rounding semantics, fp16 with prefill semantics).
// This kernel finishes the gates.
//
// Reference: fused_gates (src/rwkv_tl/kernels/gates.py:182-213) and
// fused_l2norm_neg_kk_a (src/rwkv_tl/kernels/dplr.py:45-71) on decode; the torch op
// chain of demo/_rwkv7_base.py:242-260 on prefill.
//
// grid = (M, ceil(H / 8)), block = 256: warp w handles head 8 * blockIdx.y + w of
// row blockIdx.x, lane l channels 2l, 2l+1 of the head.
#include "common.cuh"

namespace {
constexpr float kSqrtE = 1.6487212707001282f;  // sqrt(e): w = exp(-sigmoid(.)/sqrt(e))

template <typename T>
__device__ __forceinline__ float2 ld2(const T* p);
template <>
__device__ __forceinline__ float2 ld2<float>(const float* p) {
  return *reinterpret_cast<const float2*>(p);
}
template <>
__device__ __forceinline__ float2 ld2<__half>(const __half* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}
}  // namespace

template <int SEM, typename T>
__global__ void __launch_bounds__(256) k_gates_ew(
    const T* __restrict__ lora,         // 4 x [M, C]: v12, w12, a12, g12
    const __half* __restrict__ rkv,     // 3 x [M, C]: r, k, v
    const __half* __restrict__ w0, const __half* __restrict__ a0, const __half* __restrict__ v0,
    const __half* __restrict__ k_k, const __half* __restrict__ k_a,
    __half* __restrict__ vfirst,        // [M, C] written on layer 0, read otherwise
    __half* __restrict__ gout,          // 6 x [M, C]: w, k, v, A, B, g
    int M, int C, int H, int layer0) {
  RWKV_GRID_DEP_ENTRY();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int m = blockIdx.x, h = blockIdx.y * 8 + warp;
  if (h >= H) return;
  const size_t plane = (size_t)M * C;
  const int c = h * RWKV_HD + 2 * lane;
  const size_t o = (size_t)m * C + c;
  const float2 V12 = ld2<T>(lora + o), W12 = ld2<T>(lora + plane + o),
               A12 = ld2<T>(lora + 2 * plane + o), G12 = ld2<T>(lora + 3 * plane + o);
  const float2 kin = __half22float2(*reinterpret_cast<const __half2*>(rkv + plane + o));
  const float2 vin = __half22float2(*reinterpret_cast<const __half2*>(rkv + 2 * plane + o));
  float2 vf = vin;
  if (layer0)
    *reinterpret_cast<__half2*>(vfirst + o) = *reinterpret_cast<const __half2*>(rkv + 2 * plane + o);
  else
    vf = __half22float2(*reinterpret_cast<const __half2*>(vfirst + o));
  const float2 W0 = __half22float2(*reinterpret_cast<const __half2*>(w0 + c));
  const float2 A0 = __half22float2(*reinterpret_cast<const __half2*>(a0 + c));
  const float2 V0 = __half22float2(*reinterpret_cast<const __half2*>(v0 + c));
  const float2 KK = __half22float2(*reinterpret_cast<const __half2*>(k_k + c));
  const float2 KA = __half22float2(*reinterpret_cast<const __half2*>(k_a + c));
  const float v12[2] = {V12.x, V12.y}, w12[2] = {W12.x, W12.y}, a12[2] = {A12.x, A12.y},
              g12[2] = {G12.x, G12.y}, kv[2] = {kin.x, kin.y}, vv[2] = {vin.x, vin.y},
              vfv[2] = {vf.x, vf.y}, w0v[2] = {W0.x, W0.y}, a0v[2] = {A0.x, A0.y},
              v0v[2] = {V0.x, V0.y}, kkv[2] = {KK.x, KK.y}, kav[2] = {KA.x, KA.y};
  float wo[2], ko[2], vo[2], go[2], kk[2], a16[2];
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float k = kv[e], v = vv[e];
    if (SEM == SEM_DECODE) {
      vo[e] = layer0 ? v : r16(v + sigmoidf_(v0v[e] + v12[e]) * (vfv[e] - v));
      wo[e] = r16(expf(-sigmoidf_(w0v[e] + w12[e]) / kSqrtE));
      const float a = sigmoidf_(a0v[e] + a12[e]);
      a16[e] = r16(a);
      kk[e] = r16(k * kkv[e]);
      ko[e] = r16(k + kav[e] * (k * a - k));
      go[e] = r16(g12[e]);
      ss += kk[e] * kk[e];
    } else {
      vo[e] = layer0 ? v : r16(v + r16(r16(sigmoidf_(r16(v0v[e] + v12[e]))) * r16(vfv[e] - v)));
      wo[e] = r16(expf(r16(-r16(sigmoidf_(r16(w0v[e] + w12[e]))) / kSqrtE)));
      const float a = r16(sigmoidf_(r16(a0v[e] + a12[e])));
      a16[e] = a;
      kk[e] = r16(k * kkv[e]);
      ko[e] = r16(k + r16(kav[e] * r16(r16(k * a) - k)));
      go[e] = r16(g12[e]);
      ss += r16(kk[e] * kk[e]);
    }
  }
  ss = warp_sum(ss);
  float An[2], Bn[2];
  if (SEM == SEM_DECODE) {
    const float den = fmaxf(sqrtf(ss), 1e-12f);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float kn = kk[e] / den;
      An[e] = kn;
      Bn[e] = -(kn * a16[e]);
    }
  } else {
    const float den = fmaxf(r16(sqrtf(r16(ss))), 1e-12f);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float kn = r16(kk[e] / den);
      An[e] = kn;
      Bn[e] = -kn * a16[e];
    }
  }
  *reinterpret_cast<__half2*>(gout + o) = __floats2half2_rn(wo[0], wo[1]);
  *reinterpret_cast<__half2*>(gout + plane + o) = __floats2half2_rn(ko[0], ko[1]);
  *reinterpret_cast<__half2*>(gout + 2 * plane + o) = __floats2half2_rn(vo[0], vo[1]);
  *reinterpret_cast<__half2*>(gout + 3 * plane + o) = __floats2half2_rn(An[0], An[1]);
  *reinterpret_cast<__half2*>(gout + 4 * plane + o) = __floats2half2_rn(Bn[0], Bn[1]);
  *reinterpret_cast<__half2*>(gout + 5 * plane + o) = __floats2half2_rn(go[0], go[1]);
}

// `lora` is fp32 for decode semantics and fp16 for prefill semantics.
int launch_gates_ew(int sem, const void* lora, const __half* rkv, const __half* w0,
                    const __half* a0, const __half* v0, const __half* k_k, const __half* k_a,
                    __half* vfirst, __half* gout, int M, int C, int layer0, cudaStream_t st) {
  const int H = C / RWKV_HD;
  dim3 grid(M, (H + 7) / 8);
  if (sem == SEM_DECODE)
    return rwkv_launch("gates_ew", k_gates_ew<SEM_DECODE, float>, grid, dim3(256), 0, st,
                       (const float*)lora, rkv, w0, a0, v0, k_k, k_a, vfirst, gout, M, C, H, layer0);
  return rwkv_launch("gates_ew", k_gates_ew<SEM_PREFILL, __half>, grid, dim3(256), 0, st,
                     (const __half*)lora, rkv, w0, a0, v0, k_k, k_a, vfirst, gout, M, C, H, layer0);
}
