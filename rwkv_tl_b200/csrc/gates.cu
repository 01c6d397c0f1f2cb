// LoRA up-projections + gate math + per-head L2 norm, fused.
//
// Reference: fused_gates (src/rwkv_tl/kernels/gates.py:125-213) followed by
// fused_l2norm_neg_kk_a (src/rwkv_tl/kernels/dplr.py:45-71) on decode, and the
// torch op chain of demo/_rwkv7_base.py:242-260 on prefill.
//
// grid = (ceil(M/16), H), block = 256: a CTA owns 16 token rows x one head
// (64 channels), so the L2 norm over the head is CTA-local. Warp i handles
// rows 2i, 2i+1; lane l channels 2l, 2l+1. The head's slice of the packed
// up-projection [288, C] is staged in shared memory ([288][64], conflict-free
// half2 reads), the 16 rows of activated ranks in fp32.
#include "common.cuh"

namespace {
constexpr int GT_ROWS = 16;
constexpr float kSqrtE = 1.6487212707001282f;  // sqrt(e): w = exp(-sigmoid(.)/sqrt(e))
}

template <int SEM>
__global__ void __launch_bounds__(256) k_gates(
    const __half* __restrict__ ranks,   // [M, 288] v | w | a | g (fp16 GEMM outputs)
    const __half* __restrict__ w_up,    // [288, C]
    const __half* __restrict__ rkv,     // 3 x [M, C]: r, k, v
    const __half* __restrict__ w0, const __half* __restrict__ a0, const __half* __restrict__ v0,
    const __half* __restrict__ k_k, const __half* __restrict__ k_a,
    __half* __restrict__ vfirst,        // [M, C] written on layer 0, read otherwise
    __half* __restrict__ gout,          // 6 x [M, C]: w, k, v, A, B, g
    int M, int C, int layer0) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __half* sw = reinterpret_cast<__half*>(smem_raw);                      // [288][64]
  float* sr = reinterpret_cast<float*>(smem_raw + RWKV_RANK_SUM * 64 * 2);  // [16][288]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h = blockIdx.y, m_base = blockIdx.x * GT_ROWS;
  const int hc = h * RWKV_HD;

  // stage weights asynchronously: 288 rows x 128 bytes (8 x 16B chunks per row)
  for (int i = tid; i < RWKV_RANK_SUM * 8; i += 256) {
    const int j = i >> 3, q = i & 7;
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(sw + j * 64 + q * 8));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d),
                 "l"(w_up + (size_t)j * C + hc + q * 8));
  }
  asm volatile("cp.async.commit_group;\n" ::);
  // stage activated ranks (all 18 loads per thread issued before use)
  constexpr int PER = GT_ROWS * RWKV_RANK_SUM / 256;
  __half rv[PER];
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int i = tid + 256 * u;
    const int m = m_base + i / RWKV_RANK_SUM;
    rv[u] = m < M ? ranks[(size_t)m * RWKV_RANK_SUM + i % RWKV_RANK_SUM] : __float2half(0.f);
  }
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int i = tid + 256 * u;
    const int r = i / RWKV_RANK_SUM, j = i % RWKV_RANK_SUM;
    const int m = m_base + r;
    float val = 0.f;
    if (m < M) {
      val = h2f(rv[u]);
      if (j >= 32 && j < 96) {
        val = tanhf(val);
        if (SEM == SEM_PREFILL) val = r16(val);
      } else if (j >= 160) {
        val = sigmoidf_(val);
        if (SEM == SEM_PREFILL) val = r16(val);
      }
    }
    sr[i] = val;
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();

  const int r0 = 2 * warp;
  float acc[4][2][2];  // gate (v,w,a,g) x row x channel
#pragma unroll
  for (int g = 0; g < 4; ++g)
#pragma unroll
    for (int r = 0; r < 2; ++r) acc[g][r][0] = acc[g][r][1] = 0.f;

  const float* rA = sr + r0 * RWKV_RANK_SUM;
  const float* rB = rA + RWKV_RANK_SUM;
#define GATE_SEG(G, J0, J1)                                                           \
  _Pragma("unroll 8") for (int j = J0; j < J1; ++j) {                                 \
    const float2 wv = __half22float2(*reinterpret_cast<const __half2*>(sw + j * 64 + 2 * lane)); \
    const float ra = rA[j], rb = rB[j];                                               \
    acc[G][0][0] += ra * wv.x;                                                        \
    acc[G][0][1] += ra * wv.y;                                                        \
    acc[G][1][0] += rb * wv.x;                                                        \
    acc[G][1][1] += rb * wv.y;                                                        \
  }
  GATE_SEG(0, 0, 32)
  GATE_SEG(1, 32, 96)
  GATE_SEG(2, 96, 160)
  GATE_SEG(3, 160, 288)
#undef GATE_SEG

  const size_t plane = (size_t)M * C;
  const int c = hc + 2 * lane;
  const float2 W0 = __half22float2(*reinterpret_cast<const __half2*>(w0 + c));
  const float2 A0 = __half22float2(*reinterpret_cast<const __half2*>(a0 + c));
  const float2 V0 = __half22float2(*reinterpret_cast<const __half2*>(v0 + c));
  const float2 KK = __half22float2(*reinterpret_cast<const __half2*>(k_k + c));
  const float2 KA = __half22float2(*reinterpret_cast<const __half2*>(k_a + c));
  const float w0v[2] = {W0.x, W0.y}, a0v[2] = {A0.x, A0.y}, v0v[2] = {V0.x, V0.y},
              kkv[2] = {KK.x, KK.y}, kav[2] = {KA.x, KA.y};

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int m = m_base + r0 + r;
    const bool valid = m < M;  // warp-uniform
    if (!valid) continue;
    const size_t o = (size_t)m * C + c;
    const float2 kin = __half22float2(*reinterpret_cast<const __half2*>(rkv + plane + o));
    const float2 vin = __half22float2(*reinterpret_cast<const __half2*>(rkv + 2 * plane + o));
    float2 vf = vin;
    if (layer0)
      *reinterpret_cast<__half2*>(vfirst + o) = *reinterpret_cast<const __half2*>(rkv + 2 * plane + o);
    else
      vf = __half22float2(*reinterpret_cast<const __half2*>(vfirst + o));
    const float kv[2] = {kin.x, kin.y}, vv[2] = {vin.x, vin.y}, vfv[2] = {vf.x, vf.y};
    float wo[2], ko[2], vo[2], go[2], kk[2], a16[2];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float v12 = acc[0][r][e], w12 = acc[1][r][e], a12 = acc[2][r][e], g12 = acc[3][r][e];
      const float k = kv[e], v = vv[e];
      if (SEM == SEM_DECODE) {
        vo[e] = layer0 ? v : r16(v + sigmoidf_(v0v[e] + v12) * (vfv[e] - v));
        wo[e] = r16(expf(-sigmoidf_(w0v[e] + w12) / kSqrtE));
        const float a = sigmoidf_(a0v[e] + a12);
        a16[e] = r16(a);
        kk[e] = r16(k * kkv[e]);
        ko[e] = r16(k + kav[e] * (k * a - k));
        go[e] = r16(g12);
        ss += kk[e] * kk[e];
      } else {
        vo[e] = layer0 ? v
                       : r16(v + r16(r16(sigmoidf_(r16(v0v[e] + r16(v12)))) * r16(vfv[e] - v)));
        wo[e] = r16(expf(r16(-r16(sigmoidf_(r16(w0v[e] + r16(w12)))) / kSqrtE)));
        const float a = r16(sigmoidf_(r16(a0v[e] + r16(a12))));
        a16[e] = a;
        kk[e] = r16(k * kkv[e]);
        ko[e] = r16(k + r16(kav[e] * r16(r16(k * a) - k)));
        go[e] = r16(g12);
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
}

int launch_gates(int sem, const __half* ranks, const __half* w_up, const __half* rkv,
                 const __half* w0, const __half* a0, const __half* v0, const __half* k_k,
                 const __half* k_a, __half* vfirst, __half* gout, int M, int C, int layer0,
                 cudaStream_t st) {
  const size_t smem = RWKV_RANK_SUM * 64 * 2 + GT_ROWS * RWKV_RANK_SUM * 4;
  static bool attr_set[2] = {false, false};
  if (!attr_set[sem]) {
    cudaError_t e = sem == SEM_DECODE
        ? cudaFuncSetAttribute(k_gates<SEM_DECODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
        : cudaFuncSetAttribute(k_gates<SEM_PREFILL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      rwkv_set_error("gates: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return RWKV_ERR_CUDA;
    }
    attr_set[sem] = true;
  }
  dim3 grid((M + GT_ROWS - 1) / GT_ROWS, C / RWKV_HD);
  if (sem == SEM_DECODE)
    k_gates<SEM_DECODE><<<grid, 256, smem, st>>>(ranks, w_up, rkv, w0, a0, v0, k_k, k_a, vfirst,
                                                 gout, M, C, layer0);
  else
    k_gates<SEM_PREFILL><<<grid, 256, smem, st>>>(ranks, w_up, rkv, w0, a0, v0, k_k, k_a, vfirst,
                                                  gout, M, C, layer0);
  return rwkv_check_launch("gates");
}
