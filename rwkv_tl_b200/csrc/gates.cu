// Gate math + per-head L2 norm on the LoRA up-projection outputs.
//
// The up-projections themselves run as one grouped tcgen05 GEMM (gemm_tc.cu) over
// the padded rank buffer [M, 512] = v(32, zero-padded to 64) | tanh(w) hi, lo (64 + 64) | a(64) |
// sigmoid(g) hi, lo (128 + 128) and the K-major weights w_lora_up_t [C, 512], giving v12, w12, a12,
// g12 [M, C] (fp32 with decode rounding semantics, fp16 with prefill semantics).
// This kernel finishes the gates. The planes (workspace, 256-byte aligned) move in
// 16-byte accesses, 8 channels per lane.
//
// Reference: fused_gates (src/rwkv_tl/kernels/gates.py:182-213) and
// fused_l2norm_neg_kk_a (src/rwkv_tl/kernels/dplr.py:45-71) on decode; the torch op
// chain of demo/_rwkv7_base.py:242-260 on prefill.
#include "common.cuh"

namespace {
constexpr float kSqrtE = 1.6487212707001282f;  // sqrt(e): w = exp(-sigmoid(.)/sqrt(e))
}  // namespace

// N (2 or 8) consecutive channels of a workspace plane as floats.
template <int N>
__device__ __forceinline__ void ldn(const __half* p, float (&v)[N]) {
  if constexpr (N == 8) {
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
template <int N>
__device__ __forceinline__ void ldn(const float* p, float (&v)[N]) {
  if constexpr (N == 8) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const float2 a = *reinterpret_cast<const float2*>(p);
    v[0] = a.x; v[1] = a.y;
  }
}
// N channels of a per-layer weight vector (caller memory: 4-byte aligned loads).
template <int N>
__device__ __forceinline__ void ldw(const __half* p, float (&v)[N]) {
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    const float2 f = __half22float2(reinterpret_cast<const __half2*>(p)[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <int N>
__device__ __forceinline__ void stn(__half* p, const float (&v)[N]) {
  if constexpr (N == 8) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  } else {
    *reinterpret_cast<__half2*>(p) = __floats2half2_rn(v[0], v[1]);
  }
}

// grid = (M, parts of a row), block = C / VPL lanes rounded up to a warp, at most
// 256 per CTA. Each lane handles VPL consecutive channels (VPL = 8: 16-byte fp16
// accesses, for large token batches; VPL = 2 for decode-size batches, more threads per
// row); the 64 / VPL lanes of a head reduce its L2 norm together.
template <int SEM, typename T, int VPL>
__global__ void k_gates_ew(
    const T* __restrict__ lora,         // 4 x [M, C]: v12, w12, a12, g12
    const __half* __restrict__ rkv,     // 3 x [M, C]: r, k, v
    const __half* __restrict__ w0, const __half* __restrict__ a0, const __half* __restrict__ v0,
    const __half* __restrict__ k_k, const __half* __restrict__ k_a,
    __half* __restrict__ vfirst,        // [M, C] written on layer 0, read otherwise
    __half* __restrict__ gout,          // 6 x [M, C]: w, k, v, A, B, g
    int M, int C, int layer0) {
  RWKV_GRID_DEP_ENTRY();
  constexpr int P = VPL / 2;
  const int m = blockIdx.x;
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * VPL;
  const bool on = c < C;  // lanes past the row still join the group reduction
  const size_t plane = (size_t)M * C;
  const size_t o = (size_t)m * C + (on ? c : 0);
  float ssq[P], kk[VPL], a16[VPL];
#pragma unroll
  for (int q = 0; q < P; ++q) ssq[q] = 0.f;
  if (on) {
    float x[VPL], y[VPL], kin[VPL], vin[VPL], vf[VPL], out[VPL];
    ldn<VPL>(rkv + plane + o, kin);
    ldn<VPL>(rkv + 2 * plane + o, vin);
    if (layer0) {
#pragma unroll
      for (int e = 0; e < VPL; ++e) vf[e] = vin[e];
      stn<VPL>(vfirst + o, vin);  // fp16 values round-trip exactly
    } else {
      ldn<VPL>(vfirst + o, vf);
    }
    // v
    ldn<VPL>(lora + o, x);
    ldw<VPL>(v0 + c, y);
#pragma unroll
    for (int e = 0; e < VPL; ++e) {
      const float v = vin[e];
      if (layer0)
        out[e] = v;
      else if (SEM == SEM_DECODE)
        out[e] = r16(v + sigmoidf_(y[e] + x[e]) * (vf[e] - v));
      else
        out[e] = r16(v + r16(r16(sigmoidf_(r16(y[e] + x[e]))) * r16(vf[e] - v)));
    }
    stn<VPL>(gout + 2 * plane + o, out);
    // w
    ldn<VPL>(lora + plane + o, x);
    ldw<VPL>(w0 + c, y);
#pragma unroll
    for (int e = 0; e < VPL; ++e)
      out[e] = SEM == SEM_DECODE ? r16(expf(-sigmoidf_(y[e] + x[e]) / kSqrtE))
                                 : r16(expf(r16(-r16(sigmoidf_(r16(y[e] + x[e]))) / kSqrtE)));
    stn<VPL>(gout + o, out);
    // a, k, k * k_k
    ldn<VPL>(lora + 2 * plane + o, x);
    ldw<VPL>(a0 + c, y);
    float ka[VPL], kkv[VPL];
    ldw<VPL>(k_a + c, ka);
    ldw<VPL>(k_k + c, kkv);
#pragma unroll
    for (int e = 0; e < VPL; ++e) {
      const float k = kin[e];
      kk[e] = r16(k * kkv[e]);
      if (SEM == SEM_DECODE) {
        const float a = sigmoidf_(y[e] + x[e]);
        a16[e] = r16(a);
        out[e] = r16(k + ka[e] * (k * a - k));
        ssq[e / 2] += kk[e] * kk[e];
      } else {
        const float a = r16(sigmoidf_(r16(y[e] + x[e])));
        a16[e] = a;
        out[e] = r16(k + r16(ka[e] * r16(r16(k * a) - k)));
        ssq[e / 2] += r16(kk[e] * kk[e]);
      }
    }
    stn<VPL>(gout + plane + o, out);
    // g
    ldn<VPL>(lora + 3 * plane + o, x);
#pragma unroll
    for (int e = 0; e < VPL; ++e) out[e] = r16(x[e]);
    stn<VPL>(gout + 5 * plane + o, out);
  }
  const float ss = warp_sum_p<P>(ssq);
  if (!on) return;
  float An[VPL], Bn[VPL];
  if (SEM == SEM_DECODE) {
    const float den = fmaxf(sqrtf(ss), 1e-12f);
#pragma unroll
    for (int e = 0; e < VPL; ++e) {
      const float kn = kk[e] / den;
      An[e] = kn;
      Bn[e] = -(kn * a16[e]);
    }
  } else {
    const float den = fmaxf(r16(sqrtf(r16(ss))), 1e-12f);
#pragma unroll
    for (int e = 0; e < VPL; ++e) {
      const float kn = r16(kk[e] / den);
      An[e] = kn;
      Bn[e] = -kn * a16[e];
    }
  }
  stn<VPL>(gout + 3 * plane + o, An);
  stn<VPL>(gout + 4 * plane + o, Bn);
}

// `lora` is fp32 for decode semantics and fp16 for prefill semantics.
int launch_gates_ew(int sem, const void* lora, const __half* rkv, const __half* w0,
                    const __half* a0, const __half* v0, const __half* k_k, const __half* k_a,
                    __half* vfirst, __half* gout, int M, int C, int layer0, cudaStream_t st) {
  const bool wide = rwkv_rows_wide(M, 256);  // 8 channels per lane once the grid is large
  const int lanes = ((C / (wide ? 8 : 2) + 31) / 32) * 32;
  const int threads = lanes < 256 ? lanes : 256;
  const dim3 grid(M, (lanes + threads - 1) / threads), block(threads);
#define GATES_GO(S, T, V)                                                                      \
  return rwkv_launch("gates_ew", k_gates_ew<S, T, V>, grid, block, 0, st, (const T*)lora, rkv, \
                     w0, a0, v0, k_k, k_a, vfirst, gout, M, C, layer0)
  if (sem == SEM_DECODE) {
    if (wide) GATES_GO(SEM_DECODE, float, 8);
    GATES_GO(SEM_DECODE, float, 2);
  }
  if (wide) GATES_GO(SEM_PREFILL, __half, 8);
  GATES_GO(SEM_PREFILL, __half, 2);
#undef GATES_GO
}
