// wkv7 DPLR recurrence kernels.
//
// Recurrence (reference: src/rwkv_tl/kernels/dplr.py:126-227, demo/rwkv7_torch.py:49-64),
// per head, state S[v][k] fp32 64x64 (row v = value index, column k = key index):
//   sa[v]   = sum_j S[v][j] * a[j]
//   S[v][k] = S[v][k] * w[k] + sa[v] * b[k] + v[v] * k[k]
//   y[v]    = sum_k S[v][k] * r[k]
// Each row v evolves independently given the per-token vectors, so a CTA of 8
// warps owns one head: warp i keeps rows 8i..8i+7 in registers, lane l the two
// columns 2l, 2l+1 (the same 2-columns-per-lane split as the reference's
// SERIAL=2 warps), and both dot products are warp-shuffle reductions.
#include "common.cuh"

namespace {

struct TokVec {
  float2 r, w, k, a, b;
  float v[8];
};

__device__ __forceinline__ float2 ld_h2(const __half* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}

// Load the per-token vectors of one head; `base` points at column 0 of the head.
__device__ __forceinline__ void load_tok(TokVec& t, const __half* r, const __half* w,
                                         const __half* k, const __half* v, const __half* a,
                                         const __half* b, int lane, int warp) {
  const int c = 2 * lane;
  t.r = ld_h2(r + c);
  t.w = ld_h2(w + c);
  t.k = ld_h2(k + c);
  t.a = ld_h2(a + c);
  t.b = ld_h2(b + c);
  uint4 u = *reinterpret_cast<const uint4*>(v + 8 * warp);
  const __half2* hv = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(hv[i]);
    t.v[2 * i] = f.x;
    t.v[2 * i + 1] = f.y;
  }
}

// Sum 8 per-lane partials across the warp with 9 shuffles (halving exchange);
// lane l ends with the total of index (l >> 2) & 7.
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

// One recurrence step on the warp's 8 rows; y[j] (row 8*warp+j) is valid in lane 4j.
__device__ __forceinline__ void wkv_step(float2 (&s)[8], const TokVec& t, float (&y)[8]) {
  const int lane = threadIdx.x & 31;
  float p[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) p[j] = s[j].x * t.a.x + s[j].y * t.a.y;
  const float sa_mine = reduce8(p, lane);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float sa = __shfl_sync(0xffffffffu, sa_mine, 4 * j);
    s[j].x = s[j].x * t.w.x + sa * t.b.x + t.v[j] * t.k.x;
    s[j].y = s[j].y * t.w.y + sa * t.b.y + t.v[j] * t.k.y;
    p[j] = s[j].x * t.r.x + s[j].y * t.r.y;
  }
  const float y_mine = reduce8(p, lane);
#pragma unroll
  for (int j = 0; j < 8; ++j) y[j] = __shfl_sync(0xffffffffu, y_mine, 4 * j);
}

__device__ __forceinline__ void load_state(float2 (&s)[8], const float* S, int lane, int warp) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    s[j] = *reinterpret_cast<const float2*>(S + (8 * warp + j) * RWKV_HD + 2 * lane);
}
__device__ __forceinline__ void store_state(const float2 (&s)[8], float* S, int lane, int warp) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<float2*>(S + (8 * warp + j) * RWKV_HD + 2 * lane) = s[j];
}

// ---------------------------------------------------------------------------
// Standalone step / sequence kernels (the reference's fused_dplr / fused_dplr_T).
// grid = (n_seq * H), block = 256.  Vectors are [.., H, 64] fp16.
__global__ void __launch_bounds__(256) k_dplr_step(float* __restrict__ S, const __half* r,
                                                   const __half* w, const __half* k,
                                                   const __half* v, const __half* a,
                                                   const __half* b, __half* y) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const size_t head = blockIdx.x;
  float* Sh = S + head * RWKV_HD * RWKV_HD;
  const size_t off = head * RWKV_HD;
  float2 s[8];
  load_state(s, Sh, lane, warp);
  TokVec t;
  load_tok(t, r + off, w + off, k + off, v + off, a + off, b + off, lane, warp);
  float yy[8];
  wkv_step(s, t, yy);
  store_state(s, Sh, lane, warp);
  if (lane < 8) {
    float val = yy[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) val = (lane == j) ? yy[j] : val;
    y[off + 8 * warp + lane] = f2h(val);
  }
}

// grid = H, block = 256; sequential over T with one-token-ahead prefetch.
__global__ void __launch_bounds__(256) k_dplr_seq(float* __restrict__ S, const __half* r,
                                                  const __half* w, const __half* k,
                                                  const __half* v, const __half* a,
                                                  const __half* b, __half* y, int T, int H) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int h = blockIdx.x;
  float* Sh = S + (size_t)h * RWKV_HD * RWKV_HD;
  const size_t stride = (size_t)H * RWKV_HD;
  float2 s[8];
  load_state(s, Sh, lane, warp);
  TokVec cur, nxt;
  size_t off = (size_t)h * RWKV_HD;
  if (T > 0) load_tok(cur, r + off, w + off, k + off, v + off, a + off, b + off, lane, warp);
  for (int t = 0; t < T; ++t) {
    const size_t noff = off + stride;
    if (t + 1 < T) load_tok(nxt, r + noff, w + noff, k + noff, v + noff, a + noff, b + noff, lane, warp);
    float yy[8];
    wkv_step(s, cur, yy);
    if (lane < 8) {
      float val = yy[0];
#pragma unroll
      for (int j = 1; j < 8; ++j) val = (lane == j) ? yy[j] : val;
      y[off + 8 * warp + lane] = f2h(val);
    }
    cur = nxt;
    off = noff;
  }
  store_state(s, Sh, lane, warp);
}

}  // namespace

// ---------------------------------------------------------------------------
// Model wkv: recurrence + per-head GroupNorm + bonus + g gate, fused.
// grid = (n_seqs, H), block = 256. Input rows m of sequence s are consecutive.
//   rbuf  : r  [M, C]            gbuf : 6 x [M, C] = w, k, v, A(=k_hat), B, g
//   rnn   : [slots, H, 64, 64] (this layer), yg : out [M, C]
// Epilogue (warp 0, lane = channels 2l, 2l+1 of the head), see dplr.py:73-124
// (decode) and demo/_rwkv7_base.py:264-272 (prefill).
template <int SEM>
__global__ void __launch_bounds__(256) k_wkv_tokens(
    const __half* __restrict__ rbuf, const __half* __restrict__ gbuf, size_t plane,
    const __half* __restrict__ r_k, const __half* __restrict__ lnx_w,
    const __half* __restrict__ lnx_b, float* __restrict__ rnn, const int* __restrict__ cu,
    const int* __restrict__ slots, __half* __restrict__ yg, int C) {
  RWKV_GRID_DEP_ENTRY();
  __shared__ float ybuf[2][RWKV_HD];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int seq = blockIdx.x, h = blockIdx.y, H = gridDim.y;
  const int slot = slots ? slots[seq] : seq;
  float* Sh = rnn + ((size_t)slot * H + h) * RWKV_HD * RWKV_HD;
  const int m0 = cu[seq], m1 = cu[seq + 1];
  const __half *wb = gbuf, *kb = gbuf + plane, *vb = gbuf + 2 * plane, *ab = gbuf + 3 * plane,
               *bb = gbuf + 4 * plane, *gb = gbuf + 5 * plane;
  float2 s[8];
  load_state(s, Sh, lane, warp);
  const int hc = h * RWKV_HD;
  // epilogue constants for warp 0
  float2 rk = make_float2(0.f, 0.f), lw = rk, lb = rk;
  if (warp == 0) {
    rk = ld_h2(r_k + hc + 2 * lane);
    lw = ld_h2(lnx_w + hc + 2 * lane);
    lb = ld_h2(lnx_b + hc + 2 * lane);
  }
  TokVec cur, nxt;
  if (m0 < m1) {
    const size_t o = (size_t)m0 * C + hc;
    load_tok(cur, rbuf + o, wb + o, kb + o, vb + o, ab + o, bb + o, lane, warp);
  }
  int par = 0;
  for (int m = m0; m < m1; ++m) {
    if (m + 1 < m1) {
      const size_t o = (size_t)(m + 1) * C + hc;
      load_tok(nxt, rbuf + o, wb + o, kb + o, vb + o, ab + o, bb + o, lane, warp);
    }
    float yy[8];
    wkv_step(s, cur, yy);
    if (lane < 8) {
      float val = yy[0];
#pragma unroll
      for (int j = 1; j < 8; ++j) val = (lane == j) ? yy[j] : val;
      ybuf[par][8 * warp + lane] = r16(val);  // y is stored fp16 by the reference
    }
    __syncthreads();
    if (warp == 0) {
      const size_t o = (size_t)m * C + hc + 2 * lane;
      const float2 y = make_float2(ybuf[par][2 * lane], ybuf[par][2 * lane + 1]);
      const float mean = warp_sum(y.x + y.y) * (1.0f / RWKV_HD);
      const float dx = y.x - mean, dy = y.y - mean;
      const float var = warp_sum(dx * dx + dy * dy) * (1.0f / RWKV_HD);
      const float rstd = 1.0f / sqrtf(var + 64e-5f);
      const float2 rr = ld_h2(rbuf + o), kk = ld_h2(kb + o), vv = ld_h2(vb + o), gg = ld_h2(gb + o);
      float ox, oy;
      if (SEM == SEM_DECODE) {
        float p = rr.x * kk.x * rk.x;
        p += rr.y * kk.y * rk.y;
        const float rkrk = warp_sum(p);
        ox = r16(dx * rstd * lw.x + lb.x + rkrk * vv.x);
        oy = r16(dy * rstd * lw.y + lb.y + rkrk * vv.y);
      } else {
        const float fx = r16(dx * rstd * lw.x + lb.x), fy = r16(dy * rstd * lw.y + lb.y);
        const float rkrk = r16(warp_sum(r16(r16(rr.x * kk.x) * rk.x) + r16(r16(rr.y * kk.y) * rk.y)));
        ox = r16(fx + r16(rkrk * vv.x));
        oy = r16(fy + r16(rkrk * vv.y));
      }
      *reinterpret_cast<__half2*>(yg + o) = __floats2half2_rn(ox * gg.x, oy * gg.y);
    }
    cur = nxt;
    par ^= 1;
  }
  store_state(s, Sh, lane, warp);
}

template __global__ void k_wkv_tokens<SEM_DECODE>(const __half*, const __half*, size_t, const __half*,
                                                  const __half*, const __half*, float*, const int*,
                                                  const int*, __half*, int);
template __global__ void k_wkv_tokens<SEM_PREFILL>(const __half*, const __half*, size_t, const __half*,
                                                   const __half*, const __half*, float*, const int*,
                                                   const int*, __half*, int);

// One token per sequence (batched decode): grid = (n_seqs, H), 256 threads. All
// state loads of a warp are issued together and no next-token buffer is kept, so the
// kernel fits 6 CTAs per SM at 40 registers: enough bytes in flight to stream the
// 2 x 16 KiB of state per (sequence, head) at HBM rate.
struct DecVecs {
  const __half *r, *w, *k, *v, *a, *b, *g;  // [n_seqs, C] each
};

#ifndef WKV_DEC_MINB
#define WKV_DEC_MINB 6  // measured: 6 beats 5 by 1 % of the B=256 step; 7 and 8 spill (7: 13 % slower per launch, 8: 4 % on the step)
#endif
template <int SEM>
__global__ void __launch_bounds__(256, WKV_DEC_MINB) k_wkv_decode(
    const DecVecs X, const __half* __restrict__ r_k, const __half* __restrict__ lnx_w,
    const __half* __restrict__ lnx_b, float* __restrict__ rnn, const int* __restrict__ slots,
    __half* __restrict__ yg, int C) {
  RWKV_GRID_DEP_ENTRY();
  __shared__ float ybuf[RWKV_HD];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int m = blockIdx.x, h = blockIdx.y, H = gridDim.y;
  const int slot = slots ? slots[m] : m;
  float* Sh = rnn + ((size_t)slot * H + h) * RWKV_HD * RWKV_HD;
  float2 s[8];
  load_state(s, Sh, lane, warp);
  const int hc = h * RWKV_HD;
  const size_t o = (size_t)m * C + hc;
  TokVec t;
  load_tok(t, X.r + o, X.w + o, X.k + o, X.v + o, X.a + o, X.b + o, lane, warp);
  float yy[8];
  wkv_step(s, t, yy);
  store_state(s, Sh, lane, warp);
  if ((lane & 3) == 0) ybuf[8 * warp + (lane >> 2)] = r16(yy[lane >> 2]);
  __syncthreads();
  if (warp == 0) {
    const size_t oc = o + 2 * lane;
    const float2 y = make_float2(ybuf[2 * lane], ybuf[2 * lane + 1]);
    const float mean = warp_sum(y.x + y.y) * (1.0f / RWKV_HD);
    const float dx = y.x - mean, dy = y.y - mean;
    const float var = warp_sum(dx * dx + dy * dy) * (1.0f / RWKV_HD);
    const float rstd = 1.0f / sqrtf(var + 64e-5f);
    const float2 rk = ld_h2(r_k + hc + 2 * lane), lw = ld_h2(lnx_w + hc + 2 * lane),
                 lb = ld_h2(lnx_b + hc + 2 * lane);
    const float2 rr = ld_h2(X.r + oc), kk = ld_h2(X.k + oc), vv = ld_h2(X.v + oc),
                 gg = ld_h2(X.g + oc);
    float ox, oy;
    if (SEM == SEM_DECODE) {
      float p = rr.x * kk.x * rk.x;
      p += rr.y * kk.y * rk.y;
      const float rkrk = warp_sum(p);
      ox = r16(dx * rstd * lw.x + lb.x + rkrk * vv.x);
      oy = r16(dy * rstd * lw.y + lb.y + rkrk * vv.y);
    } else {
      const float fx = r16(dx * rstd * lw.x + lb.x), fy = r16(dy * rstd * lw.y + lb.y);
      const float rkrk = r16(warp_sum(r16(r16(rr.x * kk.x) * rk.x) + r16(r16(rr.y * kk.y) * rk.y)));
      ox = r16(fx + r16(rkrk * vv.x));
      oy = r16(fy + r16(rkrk * vv.y));
    }
    *reinterpret_cast<__half2*>(yg + oc) = __floats2half2_rn(ox * gg.x, oy * gg.y);
  }
}

int launch_wkv_tokens(int sem, const __half* rbuf, const __half* gbuf, size_t plane,
                      const __half* r_k, const __half* lnx_w, const __half* lnx_b, float* rnn,
                      const int* cu, const int* slots, __half* yg, int n_seqs, int H, int C,
                      cudaStream_t st) {
  dim3 grid(n_seqs, H);
  if (n_seqs * C == (int)plane) {  // one token per sequence
    const DecVecs X = {rbuf, gbuf, gbuf + plane, gbuf + 2 * plane, gbuf + 3 * plane,
                       gbuf + 4 * plane, gbuf + 5 * plane};
    return rwkv_launch("wkv_decode", sem == SEM_DECODE ? k_wkv_decode<SEM_DECODE> : k_wkv_decode<SEM_PREFILL>,
                       grid, dim3(256), 0, st, X, r_k, lnx_w, lnx_b, rnn, slots, yg, C);
  }
  return rwkv_launch("wkv_tokens", sem == SEM_DECODE ? k_wkv_tokens<SEM_DECODE> : k_wkv_tokens<SEM_PREFILL>,
                     grid, dim3(256), 0, st, rbuf, gbuf, plane, r_k, lnx_w, lnx_b, rnn, cu, slots, yg, C);
}

extern "C" int rwkv7_dplr_step(void* S, const void* r, const void* w, const void* k,
                               const void* v, const void* a, const void* b, void* y, int n_seq,
                               int H, void* stream) {
  if (!S || !r || !w || !k || !v || !a || !b || !y || n_seq < 0 || H <= 0) {
    rwkv_set_error("rwkv7_dplr_step: null pointer or bad size (n_seq=%d, H=%d)", n_seq, H);
    return RWKV_ERR_ARG;
  }
  if (n_seq == 0) return RWKV_OK;
  k_dplr_step<<<n_seq * H, 256, 0, (cudaStream_t)stream>>>(
      (float*)S, (const __half*)r, (const __half*)w, (const __half*)k, (const __half*)v,
      (const __half*)a, (const __half*)b, (__half*)y);
  return rwkv_check_launch("rwkv7_dplr_step");
}

extern "C" int rwkv7_dplr_seq(void* S, const void* r, const void* w, const void* k,
                              const void* v, const void* a, const void* b, void* y, int T, int H,
                              void* stream) {
  if (!S || !r || !w || !k || !v || !a || !b || !y || T < 0 || H <= 0) {
    rwkv_set_error("rwkv7_dplr_seq: null pointer or bad size (T=%d, H=%d)", T, H);
    return RWKV_ERR_ARG;
  }
  if (T == 0) return RWKV_OK;
  k_dplr_seq<<<H, 256, 0, (cudaStream_t)stream>>>((float*)S, (const __half*)r, (const __half*)w,
                                                  (const __half*)k, (const __half*)v,
                                                  (const __half*)a, (const __half*)b, (__half*)y,
                                                  T, H);
  return rwkv_check_launch("rwkv7_dplr_seq");
}

extern "C" int rwkv7_wkv_gn_step(void* S, const int* slots, const void* r, const void* w,
                                 const void* k, const void* v, const void* a, const void* b,
                                 const void* g, const void* r_k, const void* lnx_w,
                                 const void* lnx_b, void* out, int n_seq, int H, int semantics,
                                 void* stream) {
  if (!S || !r || !w || !k || !v || !a || !b || !g || !r_k || !lnx_w || !lnx_b || !out ||
      n_seq <= 0 || H <= 0 || (semantics != SEM_DECODE && semantics != SEM_PREFILL)) {
    rwkv_set_error("rwkv7_wkv_gn_step: null pointer or bad size (n_seq=%d, H=%d)", n_seq, H);
    return RWKV_ERR_ARG;
  }
  const int C = H * RWKV_HD;
  const DecVecs X = {(const __half*)r, (const __half*)w, (const __half*)k, (const __half*)v,
                     (const __half*)a, (const __half*)b, (const __half*)g};
  dim3 grid(n_seq, H);
  cudaStream_t st = (cudaStream_t)stream;
  if (semantics == SEM_DECODE)
    k_wkv_decode<SEM_DECODE><<<grid, 256, 0, st>>>(X, (const __half*)r_k, (const __half*)lnx_w,
                                                   (const __half*)lnx_b, (float*)S, slots,
                                                   (__half*)out, C);
  else
    k_wkv_decode<SEM_PREFILL><<<grid, 256, 0, st>>>(X, (const __half*)r_k, (const __half*)lnx_w,
                                                    (const __half*)lnx_b, (float*)S, slots,
                                                    (__half*)out, C);
  return rwkv_check_launch("rwkv7_wkv_gn_step");
}
