// Small-batch decode (B <= 8 sequences, one token each): three fused kernels per
// layer plus the head, chained with programmatic dependent launch (PDL).
//
// Reference: RWKV7Base.decode and its per-token kernels (demo/_rwkv7_base.py:74-87,
// 153-206, 276-292; src/rwkv_tl/kernels/{lerp,gates,dplr}.py) with the decode
// rounding points. At B = 1 a step streams 0.78 GB of weights, so each kernel is a
// bandwidth-bound GEMV. Everything a kernel can read before its predecessor ends --
// its weights (into registers, shared memory or L2), the token ids, the embedding
// rows and the recurrent state written by the previous step -- is read *before*
// griddepcontrol.wait, so HBM latency overlaps the previous kernel and only the
// activation hand-off stays on the critical path.
//
//   A (148 CTAs) x0 = x1 + fp16(acc2) of the previous layer (or the embedding row),
//                LN1, six token-shift mixes, GEMV over [W_rkv (3C) ; W_lora_dn (288)] rows
//   B (H CTAs)   LoRA-up + gates + L2 norm, wkv7 step on the head's fp32 state,
//                GroupNorm + bonus + g gate, then the head's 64 columns of the output
//                projection from shared memory: acc1 += W_o[:, head] @ yg (fixed-point atomics)
//   C (4C/32)    x1 = x0 + fp16(acc1), LN2, mix, 32 FFN key rows -> relu^2 ->
//                acc2 += W_fv[:, rows] @ h (fixed-point atomics)
//   head         x = x1 + fp16(acc2), ln_out, logits GEMV over V rows
// The state x of each layer is written by the kernel after the one that read it
// (every CTA of a kernel reads the old value). Workspace accumulators are zeroed
// by one memset at the start of the step, which also orders the step after the
// previous one (a plain stream dependency, not a programmatic one).
#include <cstdlib>

#include "decode_common.cuh"

namespace {

using namespace dec;

struct DecCommon {
  int B, C, H, layer;
  const int64_t* tokens;
  const int* slots;
  const __half* emb;
  __half* x0;      // [B, C] layer input
  __half* x1;      // [B, C] after TMIX
  __half* xln1;    // [B, C] LN1 output (new tmix state x)
  __half* xln2;    // [B, C] LN2 output (new cmix state x)
  __half* rkv;     // [3, B, C]
  __half* ranks;   // [B, 288]
  __half* vfirst;  // [B, C]
  long long* acc1;     // [B, C] output-projection sums of this layer, fixed point (fx_add)
  long long* acc2;     // [B, C] FFN sums of this layer (both zero on entry)
  const long long* acc2_prev;  // previous layer's FFN sums (layer > 0)
  float* rnn;      // this layer's state: [slots, H, 64, 64]
  __half* tmix_x;  // [slots, C]
  __half* cmix_x;  // [slots, C]
  __half* cmix_x_prev;  // previous layer's cmix state (written by kernel A), or null
};

__device__ __forceinline__ int slot_of(const DecCommon& P, int b) { return P.slots ? P.slots[b] : b; }

// mixes 3, 1, 4, 5). Returns the number of valid rows.
template <int RPW, int NB>
__device__ __forceinline__ int a_rows(const DecLayer& L, int C, int base, int r1, const __half* mix,
                                      const __half* (&wr)[RPW], const __half* (&xv)[RPW]) {
  int n = 0;
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int r = base + i * (NT / 32);
    int t = 0;
    const __half* wrow = L.w_rkv;
    if (r < r1) {
      n = i + 1;
      if (r < 3 * C) {
        const int part = r / C;
        t = part == 0 ? 0 : (part == 1 ? 2 : 3);
        wrow = L.w_rkv + (size_t)r * C;
      } else {
        const int j = r - 3 * C;
        t = j < 32 ? 3 : (j < 96 ? 1 : (j < 160 ? 4 : 5));
        wrow = L.w_lora_dn + (size_t)j * C;
      }
    }
    wr[i] = wrow;
    xv[i] = mix + (size_t)t * NB * C;
  }
  return n;
}

// ---------------------------------------------------------------------------
// Kernel A: x0, LN1, mixes, r/k/v + LoRA-down GEMV. grid = 148.
template <int NB, int CPL>
__global__ void __launch_bounds__(NT) k_dec_a(const DecLayer L, const DecCommon P) {
  extern __shared__ __align__(16) unsigned char smem[];
  __half* mix = reinterpret_cast<__half*>(smem);  // [6][NB][C]
  __shared__ float red[32 * 2 * NB];
  const int C = P.C, B = P.B, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rows = 3 * C + RWKV_RANK_SUM;
  const int per = (rows + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * per, r1 = min(rows, r0 + per);
  constexpr int RPW = 4;
  // ---- before the wait: weights, token rows, previous-step state
  if (tid == 0 && r0 < r1) {  // rows past the first group (rarely any) into L2
    const int a0 = r0, a1 = min(r1, 3 * C);
    if (a0 < a1) l2_prefetch_bulk(L.w_rkv + (size_t)a0 * C, (uint32_t)(a1 - a0) * C * 2);
    const int b0 = max(r0, 3 * C) - 3 * C, b1 = r1 - 3 * C;
    if (b0 < b1) l2_prefetch_bulk(L.w_lora_dn + (size_t)b0 * C, (uint32_t)(b1 - b0) * C * 2);
  }
  uint4 wpre[RPW][CPL];
  {
    const __half* wr[RPW];
    const __half* xv[RPW];
    const int n = a_rows<RPW, NB>(L, C, r0 + warp, r1, mix, wr, xv);
    gemv_load<CPL, RPW>(wr, n, lane, wpre);
  }
  float lw[CPL], lb[CPL], mu[6][CPL];
  float x[NB][CPL], prev[NB][CPL];
#pragma unroll
  for (int k = 0; k < CPL; ++k) {
    const int c = tid + NT * k;
    lw[k] = h2f(L.ln1_w[c]);
    lb[k] = h2f(L.ln1_b[c]);
#pragma unroll
    for (int t = 0; t < 6; ++t) mu[t][k] = h2f(L.mix6[t * C + c]);
  }
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int bb = b < B ? b : 0;
    const int slot = slot_of(P, bb);
    const int64_t tok = P.layer == 0 ? P.tokens[bb] : 0;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int c = tid + NT * k;
      prev[b][k] = h2f(P.tmix_x[(size_t)slot * C + c]);
      x[b][k] = P.layer == 0 ? h2f(P.emb[(size_t)tok * C + c]) : 0.f;
    }
  }
  pdl_trigger();
  pdl_wait();
  // ---- after the wait: the residual stream
  if (P.layer > 0) {
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const int bb = b < B ? b : 0;
#pragma unroll
      for (int k = 0; k < CPL; ++k) {
        const size_t o = (size_t)bb * C + tid + NT * k;
        x[b][k] = r16(h2f(P.x1[o]) + r16(fx_val(P.acc2_prev[o])));
      }
    }
  }
  if (blockIdx.x == 0) {
    for (int b = 0; b < B; ++b) {
      const int slot = slot_of(P, b);
#pragma unroll
      for (int k = 0; k < CPL; ++k) {
        const int c = tid + NT * k;
        P.x0[(size_t)b * C + c] = f2h(x[b][k]);
        // previous layer's cmix state x (its old value was read by the previous kernel)
        if (P.cmix_x_prev) P.cmix_x_prev[(size_t)slot * C + c] = P.xln2[(size_t)b * C + c];
      }
    }
  }
  ln_regs<NB, CPL>(x, lw, lb, C, red);
  // mixes (lerp.py:106-114: diff in fp16, fused fp16 fma)
#pragma unroll
  for (int b = 0; b < NB; ++b)
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int c = tid + NT * k;
      const float diff = r16(prev[b][k] - x[b][k]);
#pragma unroll
      for (int t = 0; t < 6; ++t) mix[((size_t)t * NB + b) * C + c] = f2h(x[b][k] + mu[t][k] * diff);
      if (blockIdx.x == 0 && b < B) P.xln1[(size_t)b * C + c] = f2h(x[b][k]);
    }
  __syncthreads();
  // ---- GEMV: warp rows r0 + warp + 8 i, four at a time (first group preloaded)
  for (int base = r0 + warp; base < r1; base += RPW * (NT / 32)) {
    const __half* wr[RPW];
    const __half* xv[RPW];
    const int n = a_rows<RPW, NB>(L, C, base, r1, mix, wr, xv);
    float acc[RPW][NB];
    if (base == r0 + warp) {
      gemv_dot<NB, CPL, RPW>(wpre, xv, n, C, lane, acc);
    } else {
      uint4 w[RPW][CPL];
      gemv_load<CPL, RPW>(wr, n, lane, w);
      gemv_dot<NB, CPL, RPW>(w, xv, n, C, lane, acc);
    }
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const int r = base + i * (NT / 32);
      if (i < n && lane < B) {
        float v = acc[i][0];
#pragma unroll
        for (int bb = 1; bb < NB; ++bb) v = (lane == bb) ? acc[i][bb] : v;
        if (r < 3 * C) P.rkv[((size_t)(r / C) * B + lane) * C + (r % C)] = f2h(v);
        else P.ranks[(size_t)lane * RWKV_RANK_SUM + (r - 3 * C)] = f2h(v);
      }
    }
  }
}

// Kernel B: one CTA per head: gates, wkv, GroupNorm/bonus/gate, output projection.
template <int NB>
__global__ void __launch_bounds__(NT) k_dec_b(const DecLayer L, const DecCommon P) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int C = P.C, B = P.B, h = blockIdx.x, hc = h * RWKV_HD;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __half* sw = reinterpret_cast<__half*>(smem);          // LoRA up slice [288][64]
  __half* wo = sw + RWKV_RANK_SUM * 64;                   // W_o[:, head] as [C][64]
  float* sr = reinterpret_cast<float*>(wo + (size_t)C * 64);  // activated ranks [NB][288]
  float* vec = sr + NB * RWKV_RANK_SUM;  // [7][NB][64]: r, w, k, v, A, B, g
  float* yg = vec + 7 * NB * 64;         // [NB][64]
  float* ybuf = yg + NB * 64;            // [64]
  __shared__ float lora[4][NB][64];      // v12, w12, a12, g12
  // ---- before the wait: both weight slices to shared memory, state of sequence 0
  for (int i = tid; i < RWKV_RANK_SUM * 8; i += NT) {
    const int j = i >> 3, q = i & 7;
    cp_async16(sw + j * 64 + q * 8, L.w_lora_up + (size_t)j * C + hc + q * 8);
  }
  for (int i = tid; i < C * 8; i += NT) {
    const int c = i >> 3, q = i & 7;
    // 16-byte chunk q of row c lands at chunk q ^ (c & 7): rows are 128 B apart, so
    // unswizzled, 8 consecutive rows would hit the same banks in the projection below
    cp_async16(wo + (size_t)c * 64 + ((q ^ (c & 7)) * 8), L.w_o + (size_t)c * C + hc + q * 8);
  }
  asm volatile("cp.async.commit_group;\n" ::);
  // sequence 0's state rows of this warp: written only by the previous decode step
  float2 s_pre[8];
  {
    const float* S0 = P.rnn + ((size_t)slot_of(P, 0) * P.H + h) * 64 * 64;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      s_pre[j] = *reinterpret_cast<const float2*>(S0 + (8 * warp + j) * 64 + 2 * lane);
  }
  const int c2 = hc + 2 * lane;
  const float2 W0 = __half22float2(*reinterpret_cast<const __half2*>(L.w0 + c2));
  const float2 A0 = __half22float2(*reinterpret_cast<const __half2*>(L.a0 + c2));
  const float2 V0 = __half22float2(*reinterpret_cast<const __half2*>(L.v0 + c2));
  const float2 KK = __half22float2(*reinterpret_cast<const __half2*>(L.k_k + c2));
  const float2 KA = __half22float2(*reinterpret_cast<const __half2*>(L.k_a + c2));
  const float2 RK = __half22float2(*reinterpret_cast<const __half2*>(L.r_k + c2));
  const float2 LW = __half22float2(*reinterpret_cast<const __half2*>(L.lnx_w + c2));
  const float2 LB = __half22float2(*reinterpret_cast<const __half2*>(L.lnx_b + c2));
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
  // r, k, v, v_first of this head (warp b, channels 2l, 2l+1)
  float2 rr_b = make_float2(0.f, 0.f), kin = rr_b, vin = rr_b, vf_b = rr_b;
  if (warp < B) {
    const size_t o = (size_t)warp * C + c2;
    rr_b = __half22float2(*reinterpret_cast<const __half2*>(P.rkv + o));
    kin = __half22float2(*reinterpret_cast<const __half2*>(P.rkv + (size_t)B * C + o));
    vin = __half22float2(*reinterpret_cast<const __half2*>(P.rkv + 2 * (size_t)B * C + o));
    if (P.layer > 0) vf_b = __half22float2(*reinterpret_cast<const __half2*>(P.vfirst + o));
  }
  for (int i = tid; i < 4 * NB * 64; i += NT) (&lora[0][0][0])[i] = 0.f;
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();
  {  // LoRA up: thread = (channel c, quarter of the 288 ranks); partial sums per gate
    const int c = tid & 63, qtr = tid >> 6;
    const int j0 = 72 * qtr;
    float acc[NB][4][2];
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int g = 0; g < 4; ++g) acc[b][g][0] = acc[b][g][1] = 0.f;
#pragma unroll 8
    for (int jj = 0; jj < 72; ++jj) {
      const int j = j0 + jj;
      const int g = j < 32 ? 0 : (j < 96 ? 1 : (j < 160 ? 2 : 3));
      const float wv = h2f(sw[j * 64 + c]);
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[b][g][jj & 1] += sr[b * RWKV_RANK_SUM + j] * wv;
    }
    // a quarter covers at most two gates: add only the nonzero partials (each gate's
    // sum gets at most two additions onto zero, 0 + a + b == 0 + b + a in any order,
    // so these shared-memory atomics are deterministic)
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int g0 = g == 0 ? 0 : (g == 1 ? 32 : (g == 2 ? 96 : 160));
      const int g1 = g == 0 ? 32 : (g == 1 ? 96 : (g == 2 ? 160 : 288));
      if (g1 <= j0 || g0 >= j0 + 72) continue;
#pragma unroll
      for (int b = 0; b < NB; ++b) atomicAdd(&lora[g][b][c], acc[b][g][0] + acc[b][g][1]);
    }
  }
  __syncthreads();
  // warp b: gate math + L2 norm (decode semantics, gates.py:182-213, dplr.py:45-71)
  if (warp < B) {
    const int b = warp;
    const float kv[2] = {kin.x, kin.y}, vv[2] = {vin.x, vin.y}, vfv[2] = {vf_b.x, vf_b.y},
                rv[2] = {rr_b.x, rr_b.y};
    const float w0v[2] = {W0.x, W0.y}, a0v[2] = {A0.x, A0.y}, v0v[2] = {V0.x, V0.y},
                kkv[2] = {KK.x, KK.y}, kav[2] = {KA.x, KA.y};
    float kk[2], a16[2], ss = 0.f;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int cl = 2 * lane + e;
      const float k = kv[e], v = vv[e];
      float vo;
      if (P.layer == 0) {
        vo = v;
        P.vfirst[(size_t)b * C + hc + cl] = f2h(v);
      } else {
        vo = r16(v + sigmoidf_(v0v[e] + lora[0][b][cl]) * (vfv[e] - v));
      }
      const float wd = r16(expf(-sigmoidf_(w0v[e] + lora[1][b][cl]) / 1.6487212707001282f));
      const float a = sigmoidf_(a0v[e] + lora[2][b][cl]);
      a16[e] = r16(a);
      kk[e] = r16(k * kkv[e]);
      const float ko = r16(k + kav[e] * (k * a - k));
      const int o = b * 64 + cl;
      vec[0 * NB * 64 + o] = rv[e];
      vec[1 * NB * 64 + o] = wd;
      vec[2 * NB * 64 + o] = ko;
      vec[3 * NB * 64 + o] = vo;
      vec[6 * NB * 64 + o] = r16(lora[3][b][cl]);
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
    float* Sh = P.rnn + ((size_t)slot_of(P, b) * P.H + h) * 64 * 64;
    const float* vb = vec + b * 64;
    const float2 rr = make_float2(vb[0 * NB * 64 + 2 * lane], vb[0 * NB * 64 + 2 * lane + 1]);
    const float2 ww = make_float2(vb[1 * NB * 64 + 2 * lane], vb[1 * NB * 64 + 2 * lane + 1]);
    const float2 kk = make_float2(vb[2 * NB * 64 + 2 * lane], vb[2 * NB * 64 + 2 * lane + 1]);
    const float2 aa = make_float2(vb[4 * NB * 64 + 2 * lane], vb[4 * NB * 64 + 2 * lane + 1]);
    const float2 bb = make_float2(vb[5 * NB * 64 + 2 * lane], vb[5 * NB * 64 + 2 * lane + 1]);
    float2 st[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      st[j] = b == 0 ? s_pre[j]
                     : *reinterpret_cast<const float2*>(Sh + (8 * warp + j) * 64 + 2 * lane);
    float p[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) p[j] = st[j].x * aa.x + st[j].y * aa.y;
    const float sa_mine = reduce8(p, lane);  // row 8 warp + ((lane >> 2) & 7)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float sa = __shfl_sync(0xffffffffu, sa_mine, 4 * j);
      const float v = vb[3 * NB * 64 + 8 * warp + j];
      st[j].x = st[j].x * ww.x + sa * bb.x + v * kk.x;
      st[j].y = st[j].y * ww.y + sa * bb.y + v * kk.y;
      *reinterpret_cast<float2*>(Sh + (8 * warp + j) * 64 + 2 * lane) = st[j];
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
      yg[b * 64 + 2 * lane] = r16(ox * vb[6 * NB * 64 + 2 * lane]);
      yg[b * 64 + 2 * lane + 1] = r16(oy * vb[6 * NB * 64 + 2 * lane + 1]);
    }
    __syncthreads();
  }
  // output projection over this head's 64 input columns (demo/_rwkv7_base.py:206):
  // acc1[b][c] += W_o[c, hc:hc+64] . yg[b]; thread = 4 consecutive output rows
  for (int c0 = 4 * tid; c0 < C; c0 += 4 * NT) {
    float acc[NB][4];
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[b][r] = 0.f;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int c = c0 + r;
      const uint4* wr = reinterpret_cast<const uint4*>(wo + (size_t)c * 64);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint4 w = wr[q ^ (c & 7)];
        const __half2* w2 = reinterpret_cast<const __half2*>(&w);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(w2[i]);
          const int j = q * 8 + 2 * i;
#pragma unroll
          for (int b = 0; b < NB; ++b) acc[b][r] += f.x * yg[b * 64 + j] + f.y * yg[b * 64 + j + 1];
        }
      }
    }
    for (int b = 0; b < B; ++b)
      for (int k = 0; k < 4; ++k) fx_add(P.acc1 + (size_t)b * C + c0 + k, acc[b][k]);
  }
  // new tmix state x (LN1 output) for this head's channels
  for (int i = tid; i < B * 64; i += NT) {
    const int b = i / 64, c = hc + i % 64;
    P.tmix_x[(size_t)slot_of(P, b) * C + c] = P.xln1[(size_t)b * C + c];
  }
}

// ---------------------------------------------------------------------------
// Kernel C: x1, LN2, mix, FFN over 32 hidden rows per CTA. grid = 4C / 32.
template <int NB, int CPL>
__global__ void __launch_bounds__(NT) k_dec_c(const DecLayer L, const DecCommon P) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int C = P.C, B = P.B, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __half* xk = reinterpret_cast<__half*>(smem);  // [NB][C]
  __shared__ float hbuf[NB][32];
  __shared__ float red[32 * 2 * NB];
  const int j0 = blockIdx.x * 32;
  // ---- before the wait: key rows to registers, value columns to L2, constants, state
  uint4 wkey[4][CPL];
  {
    const __half* wkr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) wkr[i] = L.w_fk + (size_t)(j0 + warp + 8 * i) * C;
    gemv_load<CPL, 4>(wkr, 4, lane, wkey);
  }
  // value slice rows c = 4 tid .. 4 tid + 3 (64 bytes each at hidden columns j0..j0+31)
  uint4 wv[4][4];
  const bool vrow = 4 * tid < C;
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (vrow)
        wv[r][u] = __ldg(reinterpret_cast<const uint4*>(L.w_fv + (size_t)(4 * tid + r) * 4 * C + j0) + u);
  float lw[CPL], lb[CPL], mu[CPL];
  float x[NB][CPL], prev[NB][CPL];
#pragma unroll
  for (int k = 0; k < CPL; ++k) {
    const int c = tid + NT * k;
    lw[k] = h2f(L.ln2_w[c]);
    lb[k] = h2f(L.ln2_b[c]);
    mu[k] = h2f(L.ffn_x_k[c]);
  }
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int slot = slot_of(P, b < B ? b : 0);
#pragma unroll
    for (int k = 0; k < CPL; ++k) prev[b][k] = h2f(P.cmix_x[(size_t)slot * C + tid + NT * k]);
  }
  pdl_trigger();
  pdl_wait();
  // ---- after the wait: x1 = x0 + fp16(acc1)
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int bb = b < B ? b : 0;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const size_t o = (size_t)bb * C + tid + NT * k;
      x[b][k] = r16(h2f(P.x0[o]) + r16(fx_val(P.acc1[o])));
      if (blockIdx.x == 0 && b < B) P.x1[o] = f2h(x[b][k]);
    }
  }
  ln_regs<NB, CPL>(x, lw, lb, C, red);
#pragma unroll
  for (int b = 0; b < NB; ++b)
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int c = tid + NT * k;
      xk[(size_t)b * C + c] = f2h(x[b][k] + mu[k] * r16(prev[b][k] - x[b][k]));
      if (blockIdx.x == 0 && b < B) P.xln2[(size_t)b * C + c] = f2h(x[b][k]);
    }
  __syncthreads();
  // 32 key rows, 4 per warp: h = relu(fp16(x . Wk))^2 in fp16
  {
    const __half* xv[4] = {xk, xk, xk, xk};
    float acc[4][NB];
    gemv_dot<NB, CPL, 4>(wkey, xv, 4, C, lane, acc);
    if (lane == 0)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const float hv = fmaxf(r16(acc[i][b]), 0.f);
          hbuf[b][warp + 8 * i] = r16(hv * hv);
        }
  }
  __syncthreads();
  // value slice: acc2[b][c] += W_fv[c, j0:j0+32] . h[b]
  if (vrow) {
    float acc[NB][4];
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[b][r] = 0.f;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const __half2* w2 = reinterpret_cast<const __half2*>(&wv[r][u]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(w2[i]);
          const int j = u * 8 + 2 * i;
#pragma unroll
          for (int b = 0; b < NB; ++b) acc[b][r] += f.x * hbuf[b][j] + f.y * hbuf[b][j + 1];
        }
      }
    for (int b = 0; b < B; ++b)
      for (int k = 0; k < 4; ++k) fx_add(P.acc2 + (size_t)b * C + 4 * tid + k, acc[b][k]);
  }
}

// ---------------------------------------------------------------------------
// Head: x = x1 + fp16(acc2), ln_out, logits = head @ x (warp per vocabulary row).
template <int NB, int CPL>
__global__ void __launch_bounds__(NT) k_dec_head(const __half* __restrict__ head,
                                                 const __half* __restrict__ lnw,
                                                 const __half* __restrict__ lnb, const DecCommon P,
                                                 int V, __half* __restrict__ logits) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int C = P.C, B = P.B, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __half* xh = reinterpret_cast<__half*>(smem);  // [NB][C]
  __shared__ float red[32 * 2 * NB];
  const int per = (V + gridDim.x - 1) / gridDim.x;
  const int v0 = blockIdx.x * per, v1 = min(V, v0 + per);
  if (tid == 0)
    for (int v = v0 + 32; v < v1; v += 32)  // beyond the preloaded first group
      l2_prefetch_bulk(head + (size_t)v * C, (uint32_t)(min(32, v1 - v) * C * 2));
  auto rows = [&](int base, const __half* (&wr)[4], const __half* (&xv)[4]) {
    int n = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int v = base + i * (NT / 32);
      if (v < v1) n = i + 1;
      wr[i] = head + (size_t)(v < v1 ? v : v0) * C;
      xv[i] = xh;
    }
    return n;
  };
  uint4 wpre[4][CPL];
  {
    const __half* wr[4];
    const __half* xv[4];
    const int n = rows(v0 + warp, wr, xv);
    gemv_load<CPL, 4>(wr, n, lane, wpre);
  }
  float lw[CPL], lb[CPL], x[NB][CPL];
#pragma unroll
  for (int k = 0; k < CPL; ++k) {
    lw[k] = h2f(lnw[tid + NT * k]);
    lb[k] = h2f(lnb[tid + NT * k]);
  }
  pdl_trigger();
  pdl_wait();
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int bb = b < B ? b : 0;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const size_t o = (size_t)bb * C + tid + NT * k;
      x[b][k] = r16(h2f(P.x1[o]) + r16(fx_val(P.acc2[o])));
    }
  }
  if (blockIdx.x == 0)
    for (int b = 0; b < B; ++b)  // last layer's cmix state x
#pragma unroll
      for (int k = 0; k < CPL; ++k) {
        const int c = tid + NT * k;
        P.cmix_x[(size_t)slot_of(P, b) * C + c] = P.xln2[(size_t)b * C + c];
      }
  ln_regs<NB, CPL>(x, lw, lb, C, red);
#pragma unroll
  for (int b = 0; b < NB; ++b)
#pragma unroll
    for (int k = 0; k < CPL; ++k) xh[(size_t)b * C + tid + NT * k] = f2h(x[b][k]);
  __syncthreads();
  for (int base = v0 + warp; base < v1; base += 4 * (NT / 32)) {
    const __half* wr[4];
    const __half* xv[4];
    const int n = rows(base, wr, xv);
    float acc[4][NB];
    if (base == v0 + warp) {
      gemv_dot<NB, CPL, 4>(wpre, xv, n, C, lane, acc);
    } else {
      uint4 w[4][CPL];
      gemv_load<CPL, 4>(wr, n, lane, w);
      gemv_dot<NB, CPL, 4>(w, xv, n, C, lane, acc);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int v = base + i * (NT / 32);
      if (i < n && lane < B) {
        float val = acc[i][0];
#pragma unroll
        for (int b = 1; b < NB; ++b) val = (lane == b) ? acc[i][b] : val;
        logits[(size_t)lane * V + v] = f2h(val);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// `pdl` false: plain stream order (the first launch of a step follows the memset and
// whatever the caller queued before it).
template <typename K, typename... Args>
int launch_pdl(bool pdl, K kernel, dim3 grid, size_t smem, cudaStream_t st, const char* name,
               Args... args) {
  // dynamic + static shared memory may exceed the default 48 KiB: always opt in
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    rwkv_set_error("%s: cudaFuncSetAttribute: %s", name, cudaGetErrorString(e));
    return RWKV_ERR_CUDA;
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
  cfg.numAttrs = pdl ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) {
    rwkv_set_error("%s: launch failed: %s", name, cudaGetErrorString(e));
    return RWKV_ERR_CUDA;
  }
  return rwkv_check_launch(name);
}

struct DecWork {
  __half *x0, *x1, *xln1, *xln2, *rkv, *ranks, *vfirst;
  long long* acc;  // [L][2][B][C], fixed point
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
  d.acc = (long long*)take((size_t)L * 2 * BC * 8);
  if (w) *w = d;
  return off;
}

template <int NB, int CPL>
int run_decode(const rwkv7_model* m, const int64_t* tokens, int B, const int* slots,
               const rwkv7_state* state, void* logits, const DecWork& w, cudaStream_t st) {
  const int L = m->n_layer, C = m->n_embd, H = C / RWKV_HD;
  const size_t BC = (size_t)B * C;
  if (cudaMemsetAsync(w.acc, 0, (size_t)L * 2 * BC * 8, st) != cudaSuccess)
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
  const size_t smem_a = 6 * (size_t)NB * C * 2;
  const size_t smem_b = RWKV_RANK_SUM * 64 * 2 + (size_t)C * 64 * 2 +
                        ((size_t)NB * RWKV_RANK_SUM + 7 * NB * 64 + NB * 64 + 64) * 4;
  const size_t smem_c = (size_t)NB * C * 2;
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
    if ((rc = launch_pdl(l > 0, k_dec_a<NB, CPL>, dim3(148), smem_a, st, "decode_gemv A", D, P)))
      return rc;
    if ((rc = launch_pdl(true, k_dec_b<NB>, dim3(H), smem_b, st, "decode_gemv B", D, P))) return rc;
    if ((rc = launch_pdl(true, k_dec_c<NB, CPL>, dim3(4 * C / 32), smem_c, st, "decode_gemv C", D, P)))
      return rc;
  }
  P.acc2 = w.acc + (size_t)(2 * L - 1) * BC;
  P.cmix_x = (__half*)state->cmix_x + (size_t)(L - 1) * ns * C;
  return launch_pdl(true, k_dec_head<NB, CPL>, dim3(296), (size_t)NB * C * 2, st, "decode_gemv head",
                    (const __half*)m->head, (const __half*)m->lnout_w, (const __half*)m->lnout_b,
                    P, m->vocab, (__half*)logits);
}

template <int CPL>
int dispatch_nb(const rwkv7_model* m, const int64_t* tokens, int B, const int* slots,
                const rwkv7_state* state, void* logits, const DecWork& w, cudaStream_t st) {
  if (B == 1) return run_decode<1, CPL>(m, tokens, B, slots, state, logits, w, st);
  if (B == 2) return run_decode<2, CPL>(m, tokens, B, slots, state, logits, w, st);
  if (B <= 4) return run_decode<4, CPL>(m, tokens, B, slots, state, logits, w, st);
  return run_decode<8, CPL>(m, tokens, B, slots, state, logits, w, st);
}

}  // namespace

int check_model_public(const rwkv7_model* m);

bool decode_persist_supported(const rwkv7_model* m, int B, const rwkv7_state* state);
size_t decode_persist_workspace(const rwkv7_model* m, int B);
int decode_persist_run(const rwkv7_model* m, const int64_t* tokens, int B, const int* slots,
                       const rwkv7_state* state, void* logits, void* ws, cudaStream_t st);

extern "C" size_t rwkv7_decode_gemv_workspace_bytes(const rwkv7_model* m, int n_seqs) {
  if (check_model_public(m) || n_seqs <= 0 || n_seqs > MAXB) return 0;
  if (m->n_embd != 768 && m->n_embd != 1024) return 0;
  const size_t a = carve_dec(nullptr, nullptr, m->n_layer, n_seqs, m->n_embd);
  const size_t b = n_seqs <= 4 ? decode_persist_workspace(m, n_seqs) : 0;
  return a > b ? a : b;
}

extern "C" int rwkv7_decode_gemv(const rwkv7_model* m, const int64_t* tokens, int n_seqs,
                                 const int* slots, const rwkv7_state* state, void* logits,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_model_public(m);
  if (rc) return rc;
  if (!tokens || !state || !state->rnn || !state->tmix_x || !state->cmix_x || !logits ||
      n_seqs <= 0 || n_seqs > MAXB || (!slots && n_seqs > state->n_slots) ||
      (m->n_embd != 768 && m->n_embd != 1024)) {
    rwkv_set_error("rwkv7_decode_gemv: bad arguments (n_seqs=%d must be 1..%d, n_embd 768 or 1024)",
                   n_seqs, MAXB);
    return RWKV_ERR_ARG;
  }
  DecWork w;
  const bool persist = decode_persist_supported(m, n_seqs, state);
  const size_t need = persist ? decode_persist_workspace(m, n_seqs)
                              : carve_dec(workspace, &w, m->n_layer, n_seqs, m->n_embd);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) {
    rwkv_set_error("rwkv7_decode_gemv: workspace needs %zu bytes, 256-aligned (got %zu)", need,
                   workspace_bytes);
    return RWKV_ERR_SPACE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  if (persist) return decode_persist_run(m, tokens, n_seqs, slots, state, logits, workspace, st);
  if (m->n_embd == 768) return dispatch_nb<3>(m, tokens, n_seqs, slots, state, logits, w, st);
  return dispatch_nb<4>(m, tokens, n_seqs, slots, state, logits, w, st);
}
