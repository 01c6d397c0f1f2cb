// Small-batch decode (B <= 8 sequences, one token each): three fused kernels per
// layer plus the head, chained with programmatic dependent launch.
//
// Reference: RWKV7Base.decode and its per-token kernels (demo/_rwkv7_base.py:74-87,
// 153-206, 276-292; src/rwkv_tl/kernels/{lerp,gates,dplr}.py) with the decode
// rounding points. At B = 1 the step is a stream of 0.78 GB of weights, so every
// kernel is a bandwidth-bound GEMV whose weight slice is prefetched into L2
// (cp.async.bulk.prefetch / prefetch.global.L2) *before* it waits on the previous
// kernel (griddepcontrol.wait): the next phase's weights stream in while the
// current phase computes, and launch gaps overlap.
//
//   A (all SMs)  x0 = x1 + fp16(acc2) of the previous layer (or the embedding row),
//                LN1, six token-shift mixes, GEMV over [W_rkv (3C) ; W_lora_dn (288)] rows
//   B (H CTAs)   LoRA-up + gates + L2 norm, wkv7 step on the head's fp32 state,
//                GroupNorm + bonus + g gate, output projection split by head:
//                acc1 += W_o[:, head] @ yg (fp32 atomics)
//   C (C/8 CTAs) x1 = x0 + fp16(acc1), LN2, mix, 32 FFN key rows -> relu^2 ->
//                acc2 += W_fv[:, rows] @ h (fp32 atomics)
//   head         x = x1 + fp16(acc2), ln_out, logits GEMV over V rows
// State x of each layer is written by the kernel after the one that read it
// (every CTA of a kernel reads the old value).
#include <cstdlib>

#include "common.cuh"

namespace {

constexpr int MAXB = 8;
constexpr int NT = 256;

struct DecLayer {
  const __half *ln1_w, *ln1_b, *ln2_w, *ln2_b, *mix6, *w_rkv, *w_lora_dn, *w_lora_up;
  const __half *w0, *a0, *v0, *k_k, *k_a, *r_k, *lnx_w, *lnx_b, *w_o, *ffn_x_k, *w_fk, *w_fv;
};

struct DecCommon {
  int B, C, H, layer;
  const int64_t* tokens;
  const int* slots;
  const __half* emb;
  // activations (workspace)
  __half* x0;      // [B, C] layer input
  __half* x1;      // [B, C] after TMIX
  __half* xln1;    // [B, C] LN1 output (new tmix state x)
  __half* xln2;    // [B, C] LN2 output (new cmix state x)
  __half* rkv;     // [3, B, C]
  __half* ranks;   // [B, 288]
  __half* vfirst;  // [B, C]
  float* acc1;     // [B, C] this layer's output-projection sum (zero on entry)
  float* acc2;     // [B, C] this layer's FFN sum (zero on entry)
  const float* acc2_prev;  // previous layer's FFN sum (layer > 0)
  // state (this layer)
  float* rnn;      // [slots, H, 64, 64]
  __half* tmix_x;  // [slots, C]
  __half* cmix_x;  // [slots, C]
  __half* cmix_x_prev;  // previous layer's cmix state (written by kernel A), or null
};

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void l2_prefetch_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void l2_prefetch_line(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
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

// Block-wide LayerNorm of NB rows of length C held in shared memory (fp32, in place),
// output rounded to fp16 like F.layer_norm on an fp16 tensor.
template <int NB>
__device__ void ln_rows_smem(float* xs, int C, const __half* w, const __half* b, float* red) {
  float s[NB];
#pragma unroll
  for (int i = 0; i < NB; ++i) s[i] = 0.f;
  for (int c = threadIdx.x; c < C; c += NT)
#pragma unroll
    for (int i = 0; i < NB; ++i) s[i] += xs[i * C + c];
  block_sum<NB>(s, red);
  float mean[NB];
#pragma unroll
  for (int i = 0; i < NB; ++i) mean[i] = s[i] / C, s[i] = 0.f;
  for (int c = threadIdx.x; c < C; c += NT)
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const float d = xs[i * C + c] - mean[i];
      s[i] += d * d;
    }
  block_sum<NB>(s, red);
  for (int c = threadIdx.x; c < C; c += NT) {
    const float ww = h2f(w[c]), bb = h2f(b[c]);
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const float rstd = rsqrtf(s[i] / C + 1e-5f);
      xs[i * C + c] = r16((xs[i * C + c] - mean[i]) * rstd * ww + bb);
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Kernel A: x0, LN1, mixes, r/k/v + LoRA-down GEMV.
template <int NB>
__global__ void __launch_bounds__(NT) k_dec_a(const DecLayer L, const DecCommon P) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int C = P.C, B = P.B;
  float* xs = reinterpret_cast<float*>(smem);                       // [NB][C] fp32
  __half* mix = reinterpret_cast<__half*>(xs + NB * C);             // [6][NB][C]
  __shared__ float red[32 * NB];
  const int rows = 3 * C + RWKV_RANK_SUM;
  const int per = (rows + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * per, r1 = min(rows, r0 + per);
  // weights of this CTA's rows into L2 while the previous kernel finishes
  if (threadIdx.x == 0 && r0 < r1) {
    const int a0 = r0, a1 = min(r1, 3 * C);
    if (a0 < a1) l2_prefetch_bulk(L.w_rkv + (size_t)a0 * C, (uint32_t)(a1 - a0) * C * 2);
    const int b0 = max(r0, 3 * C) - 3 * C, b1 = r1 - 3 * C;
    if (b0 < b1) l2_prefetch_bulk(L.w_lora_dn + (size_t)b0 * C, (uint32_t)(b1 - b0) * C * 2);
  }
  pdl_trigger();
  pdl_wait();
  // x0
  for (int i = threadIdx.x; i < NB * C; i += NT) {
    const int b = i / C, c = i % C;
    float v = 0.f;
    if (b < B) {
      if (P.layer == 0) v = h2f(P.emb[(size_t)P.tokens[b] * C + c]);
      else v = r16(h2f(P.x1[(size_t)b * C + c]) + r16(P.acc2_prev[(size_t)b * C + c]));
    }
    xs[i] = v;
    if (blockIdx.x == 0 && b < B) {
      P.x0[(size_t)b * C + c] = f2h(v);
      // previous layer's cmix state x (its old value was read by the previous kernel)
      if (P.cmix_x_prev) {
        const int slot = P.slots ? P.slots[b] : b;
        P.cmix_x_prev[(size_t)slot * C + c] = P.xln2[(size_t)b * C + c];
      }
    }
  }
  __syncthreads();
  ln_rows_smem<NB>(xs, C, L.ln1_w, L.ln1_b, red);
  // mixes (lerp.py:106-114: diff in fp16, fused fp16 fma)
  for (int i = threadIdx.x; i < NB * C; i += NT) {
    const int b = i / C, c = i % C;
    const float x = xs[i];
    float prev = 0.f;
    if (b < B) {
      const int slot = P.slots ? P.slots[b] : b;
      prev = h2f(P.tmix_x[(size_t)slot * C + c]);
      if (blockIdx.x == 0) P.xln1[(size_t)b * C + c] = f2h(x);
    }
    const float diff = r16(prev - x);
#pragma unroll
    for (int t = 0; t < 6; ++t)
      mix[((size_t)t * NB + b) * C + c] = f2h(x + h2f(L.mix6[t * C + c]) * diff);
  }
  __syncthreads();
  // GEMV: warp per row
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = r0 + warp; r < r1; r += NT / 32) {
    int t;
    const __half* wrow;
    if (r < 3 * C) {
      const int part = r / C;  // r, k, v -> mixes 0, 2, 3
      t = part == 0 ? 0 : (part == 1 ? 2 : 3);
      wrow = L.w_rkv + (size_t)r * C;
    } else {
      const int j = r - 3 * C;  // v(32) w(64) a(64) g(128) -> mixes 3, 1, 4, 5
      t = j < 32 ? 3 : (j < 96 ? 1 : (j < 160 ? 4 : 5));
      wrow = L.w_lora_dn + (size_t)j * C;
    }
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.f;
    for (int q = lane; q < C / 8; q += 32) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(wrow) + q);
#pragma unroll
      for (int b = 0; b < NB; ++b)
        acc[b] += dot8(w, reinterpret_cast<const uint4*>(mix + ((size_t)t * NB + b) * C)[q]);
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = warp_sum(acc[b]);
    if (lane < B) {
      float v = acc[0];
#pragma unroll
      for (int b = 1; b < NB; ++b) v = (lane == b) ? acc[b] : v;
      if (r < 3 * C) P.rkv[((size_t)(r / C) * B + lane) * C + (r % C)] = f2h(v);
      else P.ranks[(size_t)lane * RWKV_RANK_SUM + (r - 3 * C)] = f2h(v);
    }
  }
}

// ---------------------------------------------------------------------------
// Kernel B: per head. gates + wkv + GroupNorm/bonus/gate + output projection split.
template <int NB>
__global__ void __launch_bounds__(NT) k_dec_b(const DecLayer L, const DecCommon P) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int C = P.C, B = P.B, h = blockIdx.x, hc = h * RWKV_HD;
  __half* sw = reinterpret_cast<__half*>(smem);                                // [288][64]
  float* sr = reinterpret_cast<float*>(smem + RWKV_RANK_SUM * 64 * 2);         // [NB][288]
  float* vec = sr + NB * RWKV_RANK_SUM;  // [7][NB][64]: r, w, k, v, A, B, g
  float* yg = vec + 7 * NB * 64;         // [NB][64]
  float* ybuf = yg + NB * 64;            // [64]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // weights: LoRA-up slice to shared memory, output-projection columns to L2
  for (int i = tid; i < RWKV_RANK_SUM * 8; i += NT) {
    const int j = i >> 3, q = i & 7;
    const void* src = L.w_lora_up + (size_t)j * C + hc + q * 8;
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(sw + j * 64 + q * 8));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(src));
  }
  asm volatile("cp.async.commit_group;\n" ::);
  for (int c = tid; c < C; c += NT) l2_prefetch_line(L.w_o + (size_t)c * C + hc);
  pdl_trigger();
  pdl_wait();
  // activated ranks (gates.py:166-181: tanh for w, sigmoid for g, fp32)
  for (int i = tid; i < NB * RWKV_RANK_SUM; i += NT) {
    const int b = i / RWKV_RANK_SUM, j = i % RWKV_RANK_SUM;
    float v = b < B ? h2f(P.ranks[(size_t)b * RWKV_RANK_SUM + j]) : 0.f;
    if (j >= 32 && j < 96) v = tanhf(v);
    else if (j >= 160) v = sigmoidf_(v);
    sr[i] = v;
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();
  // warp b: LoRA-up for channels 2l, 2l+1, gate math, L2 norm (decode semantics)
  if (warp < NB && warp < B) {
    const int b = warp;
    float acc[4][2] = {};
    const float* rb = sr + b * RWKV_RANK_SUM;
#pragma unroll 4
    for (int j = 0; j < RWKV_RANK_SUM; ++j) {
      const float2 wv = __half22float2(*reinterpret_cast<const __half2*>(sw + j * 64 + 2 * lane));
      const int g = j < 32 ? 0 : (j < 96 ? 1 : (j < 160 ? 2 : 3));
      acc[g][0] += rb[j] * wv.x;
      acc[g][1] += rb[j] * wv.y;
    }
    float kk[2], a16[2], ss = 0.f;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int c = hc + 2 * lane + e;
      const float k = h2f(P.rkv[((size_t)1 * B + b) * C + c]);
      const float v = h2f(P.rkv[((size_t)2 * B + b) * C + c]);
      const float r = h2f(P.rkv[((size_t)0 * B + b) * C + c]);
      float vo;
      if (P.layer == 0) {
        vo = v;
        P.vfirst[(size_t)b * C + c] = f2h(v);
      } else {
        const float vf = h2f(P.vfirst[(size_t)b * C + c]);
        vo = r16(v + sigmoidf_(h2f(L.v0[c]) + acc[0][e]) * (vf - v));
      }
      const float wo = r16(expf(-sigmoidf_(h2f(L.w0[c]) + acc[1][e]) / 1.6487212707001282f));
      const float a = sigmoidf_(h2f(L.a0[c]) + acc[2][e]);
      a16[e] = r16(a);
      kk[e] = r16(k * h2f(L.k_k[c]));
      const float ko = r16(k + h2f(L.k_a[c]) * (k * a - k));
      const int o = b * 64 + 2 * lane + e;
      vec[0 * NB * 64 + o] = r;
      vec[1 * NB * 64 + o] = wo;
      vec[2 * NB * 64 + o] = ko;
      vec[3 * NB * 64 + o] = vo;
      vec[6 * NB * 64 + o] = r16(acc[3][e]);
      ss += kk[e] * kk[e];
    }
    ss = warp_sum(ss);
    const float den = fmaxf(sqrtf(ss), 1e-12f);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float kn = kk[e] / den;
      const int o = b * 64 + 2 * lane + e;
      vec[4 * NB * 64 + o] = r16(kn);
      vec[5 * NB * 64 + o] = r16(-(kn * a16[e]));
    }
  }
  __syncthreads();
  // wkv7 step per sequence: warp w owns state rows 8w..8w+7, lane columns 2l, 2l+1
  for (int b = 0; b < B; ++b) {
    const int slot = P.slots ? P.slots[b] : b;
    float* Sh = P.rnn + ((size_t)slot * P.H + h) * 64 * 64;
    const float* vb = vec + b * 64;
    const float2 rr = make_float2(vb[0 * NB * 64 + 2 * lane], vb[0 * NB * 64 + 2 * lane + 1]);
    const float2 ww = make_float2(vb[1 * NB * 64 + 2 * lane], vb[1 * NB * 64 + 2 * lane + 1]);
    const float2 kk = make_float2(vb[2 * NB * 64 + 2 * lane], vb[2 * NB * 64 + 2 * lane + 1]);
    const float2 aa = make_float2(vb[4 * NB * 64 + 2 * lane], vb[4 * NB * 64 + 2 * lane + 1]);
    const float2 bb = make_float2(vb[5 * NB * 64 + 2 * lane], vb[5 * NB * 64 + 2 * lane + 1]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int row = 8 * warp + j;
      float2 s = *reinterpret_cast<const float2*>(Sh + row * 64 + 2 * lane);
      float sa = s.x * aa.x;
      sa += s.y * aa.y;
      sa = warp_sum(sa);
      const float vv = vb[3 * NB * 64 + row];
      s.x = s.x * ww.x + sa * bb.x + vv * kk.x;
      s.y = s.y * ww.y + sa * bb.y + vv * kk.y;
      *reinterpret_cast<float2*>(Sh + row * 64 + 2 * lane) = s;
      float p = s.x * rr.x;
      p += s.y * rr.y;
      p = warp_sum(p);
      if (lane == 0) ybuf[row] = r16(p);
    }
    __syncthreads();
    if (warp == 0) {  // GroupNorm + bonus + g gate (dplr.py:73-124), then * g
      const float2 y = make_float2(ybuf[2 * lane], ybuf[2 * lane + 1]);
      const float mean = warp_sum(y.x + y.y) * (1.0f / 64);
      const float dx = y.x - mean, dy = y.y - mean;
      const float var = warp_sum(dx * dx + dy * dy) * (1.0f / 64);
      const float rstd = 1.0f / sqrtf(var + 64e-5f);
      const int c = hc + 2 * lane;
      const float2 rk = __half22float2(*reinterpret_cast<const __half2*>(L.r_k + c));
      const float2 lw = __half22float2(*reinterpret_cast<const __half2*>(L.lnx_w + c));
      const float2 lb = __half22float2(*reinterpret_cast<const __half2*>(L.lnx_b + c));
      float p = rr.x * kk.x * rk.x;
      p += rr.y * kk.y * rk.y;
      const float rkrk = warp_sum(p);
      const float vx = vb[3 * NB * 64 + 2 * lane], vy = vb[3 * NB * 64 + 2 * lane + 1];
      const float ox = r16(dx * rstd * lw.x + lb.x + rkrk * vx);
      const float oy = r16(dy * rstd * lw.y + lb.y + rkrk * vy);
      yg[b * 64 + 2 * lane] = r16(ox * vb[6 * NB * 64 + 2 * lane]);
      yg[b * 64 + 2 * lane + 1] = r16(oy * vb[6 * NB * 64 + 2 * lane + 1]);
    }
    __syncthreads();
  }
  // output projection, this head's 64 input columns: acc1[b][c] += W_o[c, hc:hc+64] . yg[b]
  for (int c = tid; c < C; c += NT) {
    const uint4* wr = reinterpret_cast<const uint4*>(L.w_o + (size_t)c * C + hc);
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint4 w = wr[q];
      const __half2* w2 = reinterpret_cast<const __half2*>(&w);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(w2[i]);
        const int j = q * 8 + 2 * i;
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[b] += f.x * yg[b * 64 + j] + f.y * yg[b * 64 + j + 1];
      }
    }
    for (int b = 0; b < B; ++b) atomicAdd(P.acc1 + (size_t)b * C + c, acc[b]);
  }
  // new tmix state x (LN1 output) for this head's channels
  for (int i = tid; i < B * 64; i += NT) {
    const int b = i / 64, c = hc + i % 64;
    const int slot = P.slots ? P.slots[b] : b;
    P.tmix_x[(size_t)slot * C + c] = P.xln1[(size_t)b * C + c];
  }
}

// ---------------------------------------------------------------------------
// Kernel C: x1, LN2, mix, FFN over 32 hidden rows per CTA. grid = 4C / 32.
template <int NB>
__global__ void __launch_bounds__(NT) k_dec_c(const DecLayer L, const DecCommon P) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int C = P.C, B = P.B;
  float* xs = reinterpret_cast<float*>(smem);            // [NB][C]
  __half* xk = reinterpret_cast<__half*>(xs + NB * C);   // [NB][C]
  __shared__ float hbuf[NB][32];
  __shared__ float red[32 * NB];
  const int j0 = blockIdx.x * 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) l2_prefetch_bulk(L.w_fk + (size_t)j0 * C, 32u * C * 2);
  for (int c = tid; c < C; c += NT) l2_prefetch_line(L.w_fv + (size_t)c * 4 * C + j0);
  pdl_trigger();
  pdl_wait();
  for (int i = tid; i < NB * C; i += NT) {
    const int b = i / C, c = i % C;
    float v = 0.f;
    if (b < B) v = r16(h2f(P.x0[(size_t)b * C + c]) + r16(P.acc1[(size_t)b * C + c]));
    xs[i] = v;
    if (blockIdx.x == 0 && b < B) P.x1[(size_t)b * C + c] = f2h(v);
  }
  __syncthreads();
  ln_rows_smem<NB>(xs, C, L.ln2_w, L.ln2_b, red);
  for (int i = tid; i < NB * C; i += NT) {
    const int b = i / C, c = i % C;
    const float x = xs[i];
    float prev = 0.f;
    if (b < B) {
      const int slot = P.slots ? P.slots[b] : b;
      prev = h2f(P.cmix_x[(size_t)slot * C + c]);
      if (blockIdx.x == 0) P.xln2[(size_t)b * C + c] = f2h(x);
    }
    xk[i] = f2h(x + h2f(L.ffn_x_k[c]) * r16(prev - x));
  }
  __syncthreads();
  // 32 key rows, 4 per warp: h = relu(fp16(x . Wk))^2 in fp16
  for (int jj = warp; jj < 32; jj += NT / 32) {
    const uint4* wrow = reinterpret_cast<const uint4*>(L.w_fk + (size_t)(j0 + jj) * C);
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.f;
    for (int q = lane; q < C / 8; q += 32) {
      const uint4 w = __ldg(wrow + q);
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[b] += dot8(w, reinterpret_cast<const uint4*>(xk + (size_t)b * C)[q]);
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const float hv = fmaxf(r16(warp_sum(acc[b])), 0.f);
      if (lane == 0) hbuf[b][jj] = r16(hv * hv);
    }
  }
  __syncthreads();
  // value slice: acc2[b][c] += W_fv[c, j0:j0+32] . h[b]
  for (int c = tid; c < C; c += NT) {
    const uint4* wr = reinterpret_cast<const uint4*>(L.w_fv + (size_t)c * 4 * C + j0);
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w = wr[q];
      const __half2* w2 = reinterpret_cast<const __half2*>(&w);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(w2[i]);
        const int j = q * 8 + 2 * i;
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[b] += f.x * hbuf[b][j] + f.y * hbuf[b][j + 1];
      }
    }
    for (int b = 0; b < B; ++b) atomicAdd(P.acc2 + (size_t)b * C + c, acc[b]);
  }
}

// ---------------------------------------------------------------------------
// Head: x = x1 + fp16(acc2), ln_out, logits = head @ x (warp per vocabulary row).
template <int NB>
__global__ void __launch_bounds__(NT) k_dec_head(const __half* __restrict__ head,
                                                 const __half* __restrict__ lw,
                                                 const __half* __restrict__ lb, const DecCommon P,
                                                 int V, __half* __restrict__ logits) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int C = P.C, B = P.B;
  float* xs = reinterpret_cast<float*>(smem);
  __half* xh = reinterpret_cast<__half*>(xs + NB * C);
  __shared__ float red[32 * NB];
  const int per = (V + gridDim.x - 1) / gridDim.x;
  const int v0 = blockIdx.x * per, v1 = min(V, v0 + per);
  if (threadIdx.x == 0 && v0 < v1) {
    // bulk prefetch is limited in size per instruction: issue 64 KiB pieces
    for (int v = v0; v < v1; v += 32)
      l2_prefetch_bulk(head + (size_t)v * C, (uint32_t)(min(32, v1 - v) * C * 2));
  }
  pdl_trigger();
  pdl_wait();
  for (int i = threadIdx.x; i < NB * C; i += NT) {
    const int b = i / C, c = i % C;
    float v = 0.f;
    if (b < B) v = r16(h2f(P.x1[(size_t)b * C + c]) + r16(P.acc2[(size_t)b * C + c]));
    xs[i] = v;
    if (blockIdx.x == 0 && b < B) {
      const int slot = P.slots ? P.slots[b] : b;
      P.cmix_x[(size_t)slot * C + c] = P.xln2[(size_t)b * C + c];  // last layer's cmix state
    }
  }
  __syncthreads();
  ln_rows_smem<NB>(xs, C, lw, lb, red);
  for (int i = threadIdx.x; i < NB * C; i += NT) xh[i] = f2h(xs[i]);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int v = v0 + warp; v < v1; v += NT / 32) {
    const uint4* wr = reinterpret_cast<const uint4*>(head + (size_t)v * C);
    float acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.f;
    for (int q = lane; q < C / 8; q += 32) {
      const uint4 w = __ldg(wr + q);
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[b] += dot8(w, reinterpret_cast<const uint4*>(xh + (size_t)b * C)[q]);
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = warp_sum(acc[b]);
    if (lane < B) {
      float val = acc[0];
#pragma unroll
      for (int b = 1; b < NB; ++b) val = (lane == b) ? acc[b] : val;
      logits[(size_t)lane * V + v] = f2h(val);
    }
  }
}

// ---------------------------------------------------------------------------
template <typename K, typename... Args>
int launch_pdl(K kernel, dim3 grid, size_t smem, cudaStream_t st, const char* name,
               Args... args) {
  {  // dynamic + static shared memory may exceed the default 48 KiB: always opt in
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) {
      rwkv_set_error("%s: cudaFuncSetAttribute: %s", name, cudaGetErrorString(e));
      return RWKV_ERR_CUDA;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) {
    rwkv_set_error("%s: launch failed: %s", name, cudaGetErrorString(e));
    return RWKV_ERR_CUDA;
  }
  return rwkv_check_launch(name);
}

struct DecWork {
  __half *x0, *x1, *xln1, *xln2, *rkv, *ranks, *vfirst;
  float* acc;  // [L][2][B][C]
};

size_t carve_dec(void* base, DecWork* w, int L, int B, int C) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? static_cast<char*>(base) + off : nullptr;
    off += (bytes + 255) & ~size_t(255);
    return p;
  };
  const size_t BC = (size_t)B * C;
  DecWork d;
  d.x0 = (__half*)take(BC * 2);
  d.x1 = (__half*)take(BC * 2);
  d.xln1 = (__half*)take(BC * 2);
  d.xln2 = (__half*)take(BC * 2);
  d.rkv = (__half*)take(3 * BC * 2);
  d.ranks = (__half*)take((size_t)B * RWKV_RANK_SUM * 2);
  d.vfirst = (__half*)take(BC * 2);
  d.acc = (float*)take((size_t)L * 2 * BC * 4);
  if (w) *w = d;
  return off;
}

template <int NB>
int run_decode(const rwkv7_model* m, const int64_t* tokens, int B, const int* slots,
               const rwkv7_state* state, void* logits, const DecWork& w, cudaStream_t st) {
  const int L = m->n_layer, C = m->n_embd, H = C / RWKV_HD;
  const size_t BC = (size_t)B * C;
  if (cudaMemsetAsync(w.acc, 0, (size_t)L * 2 * BC * 4, st) != cudaSuccess)
    return rwkv_check_launch("decode_gemv memset");
  DecCommon P = {};
  P.B = B;
  P.C = C;
  P.H = H;
  P.tokens = tokens;
  P.slots = slots;
  P.emb = (const __half*)m->emb;
  P.x0 = w.x0; P.x1 = w.x1; P.xln1 = w.xln1; P.xln2 = w.xln2;
  P.rkv = w.rkv; P.ranks = w.ranks; P.vfirst = w.vfirst;
  const int ns = state->n_slots;
  const size_t smem_a = (size_t)NB * C * 4 + 6 * (size_t)NB * C * 2;
  const size_t smem_b = RWKV_RANK_SUM * 64 * 2 + (size_t)NB * RWKV_RANK_SUM * 4 +
                        (7 * NB * 64 + NB * 64 + 64) * 4;
  const size_t smem_c = (size_t)NB * C * 4 + (size_t)NB * C * 2;
  int rc;
  for (int l = 0; l < L; ++l) {
    const rwkv7_layer& s = m->layers[l];
    DecLayer D = {(const __half*)s.ln1_w, (const __half*)s.ln1_b, (const __half*)s.ln2_w,
                  (const __half*)s.ln2_b, (const __half*)s.mix6, (const __half*)s.w_rkv,
                  (const __half*)s.w_lora_dn, (const __half*)s.w_lora_up, (const __half*)s.w0,
                  (const __half*)s.a0, (const __half*)s.v0, (const __half*)s.k_k,
                  (const __half*)s.k_a, (const __half*)s.r_k, (const __half*)s.lnx_w,
                  (const __half*)s.lnx_b, (const __half*)s.w_o, (const __half*)s.ffn_x_k,
                  (const __half*)s.w_fk, (const __half*)s.w_fv};
    P.layer = l;
    P.acc1 = w.acc + (size_t)(2 * l) * BC;
    P.acc2 = w.acc + (size_t)(2 * l + 1) * BC;
    P.acc2_prev = l ? w.acc + (size_t)(2 * l - 1) * BC : nullptr;
    P.rnn = (float*)state->rnn + (size_t)l * ns * H * 4096;
    P.tmix_x = (__half*)state->tmix_x + (size_t)l * ns * C;
    P.cmix_x = (__half*)state->cmix_x + (size_t)l * ns * C;
    P.cmix_x_prev = l ? (__half*)state->cmix_x + (size_t)(l - 1) * ns * C : nullptr;
    if ((rc = launch_pdl(k_dec_a<NB>, dim3(148), smem_a, st, "decode_gemv A", D, P))) return rc;
    if ((rc = launch_pdl(k_dec_b<NB>, dim3(H), smem_b, st, "decode_gemv B", D, P))) return rc;
    if ((rc = launch_pdl(k_dec_c<NB>, dim3(4 * C / 32), smem_c, st, "decode_gemv C", D, P)))
      return rc;
  }
  P.acc2 = w.acc + (size_t)(2 * L - 1) * BC;
  P.cmix_x = (__half*)state->cmix_x + (size_t)(L - 1) * ns * C;
  const size_t smem_h = (size_t)NB * C * 4 + (size_t)NB * C * 2;
  return launch_pdl(k_dec_head<NB>, dim3(296), smem_h, st, "decode_gemv head",
                    (const __half*)m->head, (const __half*)m->lnout_w, (const __half*)m->lnout_b,
                    P, m->vocab, (__half*)logits);
}

}  // namespace

int check_model_public(const rwkv7_model* m);

extern "C" size_t rwkv7_decode_gemv_workspace_bytes(const rwkv7_model* m, int n_seqs) {
  if (check_model_public(m) || n_seqs <= 0 || n_seqs > MAXB) return 0;
  return carve_dec(nullptr, nullptr, m->n_layer, n_seqs, m->n_embd);
}

extern "C" int rwkv7_decode_gemv(const rwkv7_model* m, const int64_t* tokens, int n_seqs,
                                 const int* slots, const rwkv7_state* state, void* logits,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_model_public(m);
  if (rc) return rc;
  if (!tokens || !state || !state->rnn || !state->tmix_x || !state->cmix_x || !logits ||
      n_seqs <= 0 || n_seqs > MAXB || (!slots && n_seqs > state->n_slots) ||
      m->n_embd % 256) {
    rwkv_set_error("rwkv7_decode_gemv: bad arguments (n_seqs=%d must be 1..%d, n_embd %% 256 == 0)",
                   n_seqs, MAXB);
    return RWKV_ERR_ARG;
  }
  DecWork w;
  const size_t need = carve_dec(workspace, &w, m->n_layer, n_seqs, m->n_embd);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) {
    rwkv_set_error("rwkv7_decode_gemv: workspace needs %zu bytes, 256-aligned (got %zu)", need,
                   workspace_bytes);
    return RWKV_ERR_SPACE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  if (n_seqs == 1) return run_decode<1>(m, tokens, n_seqs, slots, state, logits, w, st);
  if (n_seqs == 2) return run_decode<2>(m, tokens, n_seqs, slots, state, logits, w, st);
  if (n_seqs <= 4) return run_decode<4>(m, tokens, n_seqs, slots, state, logits, w, st);
  return run_decode<8>(m, tokens, n_seqs, slots, state, logits, w, st);
}
