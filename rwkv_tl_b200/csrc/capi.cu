// C-ABI entry points: error reporting and the token-batch forward driver.
//
// rwkv7_forward runs the layer loop of RWKV7Base.prefill / decode
// (demo/_rwkv7_base.py:74-98) for a batch of token rows of many sequences:
// per layer TMIX (row LN+shift+mix -> r/k/v GEMM -> LoRA-down GEMM -> gates ->
// wkv+GroupNorm+gate -> output GEMM + residual) and CMIX (row LN+shift+mix ->
// key GEMM + relu^2 -> value GEMM + residual), then ln_out + head GEMM for the
// requested rows and the state-x write-back.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>

#include "common.cuh"

static thread_local char g_err[512] = "";

void rwkv_set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

static unsigned long long g_launches = 0;  // kernels launched by this library (host side)

int rwkv_check_launch(const char* what) {
  __atomic_add_fetch(&g_launches, 1ull, __ATOMIC_RELAXED);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    rwkv_set_error("%s: CUDA error %s", what, cudaGetErrorString(e));
    return RWKV_ERR_CUDA;
  }
  return RWKV_OK;
}

extern "C" const char* rwkv_b200_last_error(void) { return g_err; }
extern "C" int rwkv_b200_abi_version(void) { return RWKV_B200_ABI_VERSION; }
int gemm_tc_timeout_flag();
bool rwkv_pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("RWKV_B200_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

namespace {
thread_local bool t_chain_first = true;
}
void rwkv_chain_begin() { t_chain_first = true; }
bool rwkv_chain_take_pdl() {
  const bool first = t_chain_first;
  t_chain_first = false;
  return !first && rwkv_pdl_enabled();
}

bool rwkv_rows_wide(int M, int C) {
  const char* e = getenv("RWKV_B200_NARROW");
  if (e && e[0] == '1') return false;
  return M >= 1024 && C % 256 == 0;
}

int decode_persist_timeout_flag();
int wkv_chunk_bad_flag();
extern "C" int rwkv_b200_device_error(void) {
  const int a = gemm_tc_timeout_flag() != 0, b = decode_persist_timeout_flag() != 0,
            c = wkv_chunk_bad_flag() != 0;
  return a | (b << 1) | (c << 2);
}

int wait_selftest_tc(int* out, cudaStream_t st);
int wait_selftest_persist(void* bar, int* out, cudaStream_t st);
int wait_selftest_scan(int* out, cudaStream_t st);
extern "C" int rwkv_b200_wait_selftest(int which, void* scratch, void* stream) {
  rwkv_chain_begin();
  if (!scratch || (reinterpret_cast<uintptr_t>(scratch) & 15)) {
    rwkv_set_error("rwkv_b200_wait_selftest: scratch must be 32 zeroed, 16-byte aligned bytes");
    return RWKV_ERR_ARG;
  }
  int* out = reinterpret_cast<int*>(static_cast<char*>(scratch) + 16);
  cudaStream_t st = (cudaStream_t)stream;
  switch (which) {
    case 0: return wait_selftest_tc(out, st);
    case 1: return wait_selftest_persist(scratch, out, st);
    case 2: return wait_selftest_scan(out, st);
    default:
      rwkv_set_error("rwkv_b200_wait_selftest: which must be 0, 1 or 2 (got %d)", which);
      return RWKV_ERR_ARG;
  }
}

extern "C" unsigned long long rwkv_b200_launch_count(void) {
  return __atomic_load_n(&g_launches, __ATOMIC_RELAXED);
}

// launchers from the other translation units
int launch_tmix_rows(int sem, __half* x, const int64_t* tokens, const __half* emb,
                     const __half* ln_w, const __half* ln_b, const __half* mix6,
                     const __half* state_x, const int* row_seq, const int* cu, const int* slots,
                     __half* xmix, __half* xlast, int M, int C, PendingResid pend,
                     cudaStream_t st);
int launch_cmix_rows(int sem, __half* x, const __half* ln_w, const __half* ln_b,
                     const __half* mu, const __half* state_x, const int* row_seq, const int* cu,
                     const int* slots, __half* xk, __half* xlast, int M, int C, PendingResid pend,
                     cudaStream_t st);
int launch_ln_rows(const __half* x, const int* rows, const __half* w, const __half* b,
                   __half* out, int n, int M, int C, PendingResid pend, cudaStream_t st);
int launch_argmax_finish(const unsigned long long* keys, int64_t* ids, int n, cudaStream_t st);
int launch_scatter_state_x(const __half* xlast, __half* tmix_x, __half* cmix_x, const int* slots,
                           int S, int L, int n_slots, int C, cudaStream_t st);
int launch_gates_ew(int sem, const void* lora, const __half* rkv, const __half* w0,
                    const __half* a0, const __half* v0, const __half* k_k, const __half* k_a,
                    __half* vfirst, __half* gout, int M, int C, int layer0, cudaStream_t st);
int launch_wkv_tokens(int sem, const __half* rbuf, const __half* gbuf, size_t plane,
                      const __half* r_k, const __half* lnx_w, const __half* lnx_b, float* rnn,
                      const int* cu, const int* slots, __half* yg, int n_seqs, int H, int C,
                      cudaStream_t st);
int gemm_launch_ws(const rwkv7_gemm_problem* problems, int n, int epi, float* ws,
                   size_t ws_floats, cudaStream_t st, int* splits_out = nullptr);
size_t wkv_chunk_record_bytes(int M, int S, int H);
int launch_chunk_table(const int* cu, int* chunk_cu, float* rec, int M, int S, int H,
                       cudaStream_t st);
int launch_wkv_chunked(const __half* r, const __half* w, const __half* k, const __half* v,
                       const __half* a, const __half* b, float* rnn, const int* cu,
                       const int* slots, __half* ybuf, float* rec, int* chunk_cu, int M, int S,
                       int H, int n_slots, cudaStream_t st);
int launch_wkv_epilogue(int sem, const __half* ybuf, const __half* rbuf, const __half* gbuf,
                        size_t plane, const __half* r_k, const __half* lnx_w,
                        const __half* lnx_b, __half* yg, int M, int C, cudaStream_t st);

namespace {

struct Carve {
  char* base;
  size_t off = 0;
  explicit Carve(void* b) : base(static_cast<char*>(b)) {}
  template <typename T>
  T* take(size_t count) {
    T* p = reinterpret_cast<T*>(base ? base + off : nullptr);
    off += (count * sizeof(T) + 255) & ~size_t(255);
    return p;
  }
};

// rank buffer columns: v(32) | 0(32) | w hi(64) | w lo(64) | a(64) | g hi(128) | g lo(128);
// the lo parts carry fp32 activations exactly for the decode semantics (zero for prefill)
constexpr int RANKS_LD = 512;

struct Work {
  __half *x, *x1, *xmix, *rkv, *ranks, *gbuf, *vfirst, *yg, *xk, *h, *xlast, *lnout;
  void* lora;  // 4 x [M, C] LoRA up outputs (fp32 decode semantics, fp16 prefill)
  float* chunk_rec;
  int* chunk_cu;
  unsigned long long* argmax_keys;  // [n_logits] greedy-head keys (zero between calls)
  float* splitk;       // split-K partial tiles for small-M GEMMs
  size_t splitk_floats;
  float* splitk_side;  // the same for the r/k/v GEMM on the side stream (decode batches)
};

// token batches of at most this many rows run r/k/v on a side stream (measured: no gain
// for prefill-sized batches, whose GEMMs fill the GPU by themselves)
constexpr int kForkMaxRows = 512;

// split-K only pays for small token batches
size_t splitk_floats(int M, int C) { return M <= 1024 ? (size_t)16 * M * C : 0; }

// Side stream for the r/k/v projections of small token batches (decode): those GEMMs
// fill only part of the GPU (one 128 x 64 tile per CTA, one CTA per SM) and nothing but
// the gate kernel reads their output, so they run beside the LoRA chain (down, reduce,
// up) instead of before it. One non-blocking stream and two events per device and host
// thread (calls from different threads never share an event, so their fork / join points
// cannot cross), created on the thread's first such call that is not being captured into
// a CUDA graph (a call captured before them runs on the caller's stream alone, with the
// same results); RWKV_B200_FORK=0 keeps everything on the caller's stream.
struct ForkRes {
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  bool ok = false;
};
ForkRes* fork_res(cudaStream_t st) {
  const char* e = std::getenv("RWKV_B200_FORK");
  if (e && e[0] == '0') return nullptr;
  static thread_local ForkRes res[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  ForkRes& r = res[dev];
  if (!r.ok && !r.side) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
      return nullptr;  // create nothing inside a capture
    if (cudaStreamCreateWithFlags(&r.side, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&r.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&r.join, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      r.side = reinterpret_cast<cudaStream_t>(1);  // do not retry; stay on one stream
      return nullptr;
    }
    r.ok = true;
  }
  return r.ok ? &r : nullptr;
}

// The chunk-parallel wkv pays off once sequences are long; one-token rows
// (decode) use the fused per-token kernel. RWKV_B200_WKV=serial|chunked forces one.
bool use_chunked_wkv(int M, int S) {
  const char* e = getenv("RWKV_B200_WKV");
  if (e && e[0] == 's') return false;
  if (e && e[0] == 'c') return true;
  return M >= 32 * S;
}

Work carve(void* base, size_t& total, int M, int S, int L, int C, int n_logits) {
  Carve c(base);
  const size_t MC = (size_t)M * C;
  Work w;
  w.x = c.take<__half>(MC);
  w.x1 = c.take<__half>(MC);
  w.xmix = c.take<__half>(6 * MC);
  w.rkv = c.take<__half>(3 * MC);
  w.ranks = c.take<__half>((size_t)M * RANKS_LD);
  w.lora = c.take<float>(4 * MC);
  w.gbuf = c.take<__half>(6 * MC);
  w.vfirst = c.take<__half>(MC);
  w.yg = c.take<__half>(MC);
  w.xk = c.take<__half>(MC);
  w.h = c.take<__half>(4 * MC);
  w.xlast = c.take<__half>((size_t)L * 2 * S * C);
  w.lnout = c.take<__half>((size_t)n_logits * C);
  w.argmax_keys = c.take<unsigned long long>((size_t)n_logits);
  w.chunk_cu = c.take<int>((size_t)S + 1);
  w.chunk_rec = c.take<float>(wkv_chunk_record_bytes(M, S, C / RWKV_HD) / sizeof(float));
  w.splitk_floats = splitk_floats(M, C);
  w.splitk = w.splitk_floats ? c.take<float>(w.splitk_floats) : nullptr;
  // a region of its own, as large, so the side-stream r/k/v GEMM splits exactly as it
  // would on the caller's stream (same K-slices, same sums)
  w.splitk_side = M <= kForkMaxRows && w.splitk_floats ? c.take<float>(w.splitk_floats) : nullptr;
  total = c.off;
  return w;
}

int check_model(const rwkv7_model* m) {
  if (!m || !m->layers || !m->emb || !m->head || m->n_layer <= 0 || !m->layers[0].w_lora_up_t) {
    rwkv_set_error("rwkv7_model: null pointer or no layers");
    return RWKV_ERR_ARG;
  }
  if (m->n_embd % 128 || m->n_embd < 128 || m->n_embd > 4096) {
    rwkv_set_error("rwkv7_model: n_embd must be a multiple of 128 in [128, 4096] (got %d)",
                   m->n_embd);
    return RWKV_ERR_ARG;
  }
  if (m->rank_v != RWKV_RANK_V || m->rank_w != RWKV_RANK_W || m->rank_a != RWKV_RANK_A ||
      m->rank_g != RWKV_RANK_G) {
    rwkv_set_error("rwkv7_model: LoRA ranks must be v=32 w=64 a=64 g=128 (got %d %d %d %d)",
                   m->rank_v, m->rank_w, m->rank_a, m->rank_g);
    return RWKV_ERR_ARG;
  }
  if (m->vocab <= 0 || m->vocab % 2) {
    rwkv_set_error("rwkv7_model: vocab must be positive and even (got %d)", m->vocab);
    return RWKV_ERR_ARG;
  }
  return RWKV_OK;
}

#define TRY(expr)         \
  do {                    \
    int _rc = (expr);     \
    if (_rc) return _rc;  \
  } while (0)

}  // namespace

int check_model_public(const rwkv7_model* m) { return check_model(m); }

extern "C" size_t rwkv7_forward_workspace_bytes(const rwkv7_model* model, int n_rows, int n_seqs,
                                                int n_logits) {
  if (check_model(model) || n_rows < 0 || n_seqs < 0 || n_logits < 0) return 0;
  size_t total = 0;
  carve(nullptr, total, n_rows, n_seqs, model->n_layer, model->n_embd, n_logits);
  return total;
}

extern "C" int rwkv7_forward(const rwkv7_model* model, const rwkv7_batch* b,
                             const rwkv7_state* state, void* workspace, size_t workspace_bytes,
                             void* stream) {
  TRY(check_model(model));
  if (!b || !state || !state->rnn || !state->tmix_x || !state->cmix_x) {
    rwkv_set_error("rwkv7_forward: null batch/state");
    return RWKV_ERR_ARG;
  }
  const int M = b->n_rows, S = b->n_seqs, L = model->n_layer, C = model->n_embd, H = C / RWKV_HD;
  if (M <= 0 || S <= 0 || S > M || !b->tokens || !b->cu_seqlens || !b->row_seq ||
      b->n_logits < 0 || (b->n_logits && (!b->logit_rows || (!b->logits && !b->next_ids))) ||
      (b->semantics != RWKV_SEM_DECODE && b->semantics != RWKV_SEM_PREFILL) ||
      (!b->slots && S > state->n_slots)) {
    rwkv_set_error("rwkv7_forward: bad batch (rows=%d seqs=%d logits=%d semantics=%d)", M, S,
                   b->n_logits, b->semantics);
    return RWKV_ERR_ARG;
  }
  if ((size_t)M * 4 * C > ((size_t)1 << 31)) {
    rwkv_set_error("rwkv7_forward: too many rows in one call (%d); split the batch", M);
    return RWKV_ERR_ARG;
  }
  size_t need = 0;
  Work w = carve(workspace, need, M, S, L, C, b->n_logits);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) {
    rwkv_set_error("rwkv7_forward: workspace needs %zu bytes, 256-aligned (got %zu)", need,
                   workspace_bytes);
    return RWKV_ERR_SPACE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const int sem = b->semantics;
  const size_t MC = (size_t)M * C;
  const size_t CC = (size_t)C * C;
  const int ns = state->n_slots;
  const __half* emb = (const __half*)model->emb;
  const bool chunked = use_chunked_wkv(M, S);
  // r/k/v beside the LoRA chain only while both fit on the GPU at once (decode batches)
  ForkRes* fk = M <= kForkMaxRows && w.splitk_side ? fork_res(st) : nullptr;
  rwkv_chain_begin();
  // columns 32..63 of the rank buffer (the zero padding of rank v) must read as zero
  if (cudaMemsetAsync(w.ranks, 0, (size_t)M * RANKS_LD * sizeof(__half), st) != cudaSuccess)
    return rwkv_check_launch("ranks memset");

  // The residual GEMMs (W_o, FFN value) leave a split-K reduce to the next row kernel
  // (cmix_rows / the next layer's tmix_rows / ln_rows), which needs the sum anyway.
  PendingResid pend{nullptr, nullptr, 0};
  auto defer = [&](int splits, const __half* res) {
    pend = splits > 1 ? PendingResid{w.splitk, res, splits} : PendingResid{nullptr, nullptr, 0};
  };
  if (chunked) TRY(launch_chunk_table(b->cu_seqlens, w.chunk_cu, w.chunk_rec, M, S, H, st));
  for (int l = 0; l < L; ++l) {
    const rwkv7_layer& Lw = model->layers[l];
    const __half* wrkv = (const __half*)Lw.w_rkv;
    const __half* wdn = (const __half*)Lw.w_lora_dn;
    __half* st_tx = (__half*)state->tmix_x + (size_t)l * ns * C;
    __half* st_cx = (__half*)state->cmix_x + (size_t)l * ns * C;
    float* st_rnn = (float*)state->rnn + (size_t)l * ns * H * RWKV_HD * RWKV_HD;
    __half* xl_t = w.xlast + ((size_t)l * 2 + 0) * S * C;
    __half* xl_c = w.xlast + ((size_t)l * 2 + 1) * S * C;

    // ---- TMIX ----
    TRY(launch_tmix_rows(sem, w.x, l == 0 ? b->tokens : nullptr, emb, (const __half*)Lw.ln1_w,
                         (const __half*)Lw.ln1_b, (const __half*)Lw.mix6, st_tx, b->row_seq,
                         b->cu_seqlens, b->slots, w.xmix, xl_t, M, C, pend, st));
    {
      // r/k/v projections: xmix planes r=0, k=2, v=3
      rwkv7_gemm_problem p[3] = {
          {w.xmix + 0 * MC, wrkv + 0 * CC, w.rkv + 0 * MC, nullptr, M, C, C, C, C, C},
          {w.xmix + 2 * MC, wrkv + 1 * CC, w.rkv + 1 * MC, nullptr, M, C, C, C, C, C},
          {w.xmix + 3 * MC, wrkv + 2 * CC, w.rkv + 2 * MC, nullptr, M, C, C, C, C, C}};
      if (fk) {
        if (cudaEventRecord(fk->fork, st) != cudaSuccess ||
            cudaStreamWaitEvent(fk->side, fk->fork, 0) != cudaSuccess)
          return rwkv_check_launch("fork");
        rwkv_chain_begin();  // plain launch on the side stream
        TRY(gemm_launch_ws(p, 3, RWKV_EPI_STORE, w.splitk_side, w.splitk_floats, fk->side));
        if (cudaEventRecord(fk->join, fk->side) != cudaSuccess) return rwkv_check_launch("join");
        // the LoRA-down keeps its programmatic edge to the row kernel
      } else
        TRY(gemm_launch_ws(p, 3, RWKV_EPI_STORE, w.splitk, w.splitk_floats, st));
    }
    {
      // LoRA down-projections into the rank buffer: v, tanh(w), a, sigmoid(g), activations
      // applied on the fp16-rounded GEMM outputs (decode: fp32 activation as hi + lo)
      const int R = RANKS_LD;
      rwkv7_gemm_problem p[4] = {
          {w.xmix + 3 * MC, wdn + 0 * C, w.ranks + 0, nullptr, M, 32, C, C, C, R},
          {w.xmix + 1 * MC, wdn + 32 * C, w.ranks + 64, nullptr, M, 64, C, C, C, R},
          {w.xmix + 4 * MC, wdn + 96 * C, w.ranks + 192, nullptr, M, 64, C, C, C, R},
          {w.xmix + 5 * MC, wdn + 160 * C, w.ranks + 256, nullptr, M, 128, C, C, C, R}};
      TRY(gemm_launch_ws(p, 4, sem == SEM_DECODE ? RWKV_EPI_LORA_ACT2 : RWKV_EPI_LORA_ACT,
                         w.splitk, w.splitk_floats, st));
    }
    {
      // LoRA up-projections on tensor cores: v12, w12, a12, g12 [M, C]
      const int R = RANKS_LD;
      const __half* up = (const __half*)Lw.w_lora_up_t;
      const bool f32 = sem == SEM_DECODE;
      const size_t esz = f32 ? 4 : 2;
      char* lo = (char*)w.lora;
      rwkv7_gemm_problem p[4] = {
          {w.ranks + 0, up + 0, lo + 0 * MC * esz, nullptr, M, C, 64, R, R, C},
          {w.ranks + 64, up + 64, lo + 1 * MC * esz, nullptr, M, C, 128, R, R, C},
          {w.ranks + 192, up + 192, lo + 2 * MC * esz, nullptr, M, C, 64, R, R, C},
          {w.ranks + 256, up + 256, lo + 3 * MC * esz, nullptr, M, C, 256, R, R, C}};
      TRY(gemm_launch_ws(p, 4, f32 ? RWKV_EPI_STORE_F32 : RWKV_EPI_STORE, w.splitk,
                         w.splitk_floats, st));
    }
    if (fk) {
      if (cudaStreamWaitEvent(st, fk->join, 0) != cudaSuccess) return rwkv_check_launch("join");
      rwkv_chain_begin();  // the gate kernel waits for the side stream in full
    }
    TRY(launch_gates_ew(sem, w.lora, w.rkv, (const __half*)Lw.w0, (const __half*)Lw.a0,
                        (const __half*)Lw.v0, (const __half*)Lw.k_k, (const __half*)Lw.k_a,
                        w.vfirst, w.gbuf, M, C, l == 0, st));
    if (chunked) {
      // gbuf planes: 0 w, 1 k, 2 v, 3 A (k_hat), 4 B; r from the rkv buffer
      TRY(launch_wkv_chunked(w.rkv, w.gbuf, w.gbuf + MC, w.gbuf + 2 * MC, w.gbuf + 3 * MC,
                             w.gbuf + 4 * MC, st_rnn, b->cu_seqlens, b->slots, w.xk, w.chunk_rec,
                             w.chunk_cu, M, S, H, ns, st));
      TRY(launch_wkv_epilogue(sem, w.xk, w.rkv, w.gbuf, MC, (const __half*)Lw.r_k,
                              (const __half*)Lw.lnx_w, (const __half*)Lw.lnx_b, w.yg, M, C, st));
    } else
      TRY(launch_wkv_tokens(sem, w.rkv, w.gbuf, MC, (const __half*)Lw.r_k,
                            (const __half*)Lw.lnx_w, (const __half*)Lw.lnx_b, st_rnn,
                            b->cu_seqlens, b->slots, w.yg, S, H, C, st));
    {
      rwkv7_gemm_problem p = {w.yg, Lw.w_o, w.x1, w.x, M, C, C, C, C, C};
      int splits = 1;
      TRY(gemm_launch_ws(&p, 1, RWKV_EPI_RESID, w.splitk, w.splitk_floats, st, &splits));
      defer(splits, w.x);
    }
    // ---- CMIX ----
    TRY(launch_cmix_rows(sem, w.x1, (const __half*)Lw.ln2_w, (const __half*)Lw.ln2_b,
                         (const __half*)Lw.ffn_x_k, st_cx, b->row_seq, b->cu_seqlens, b->slots,
                         w.xk, xl_c, M, C, pend, st));
    {
      rwkv7_gemm_problem p = {w.xk, Lw.w_fk, w.h, nullptr, M, 4 * C, C, C, C, 4 * C};
      TRY(gemm_launch_ws(&p, 1, RWKV_EPI_RELUSQ, w.splitk, w.splitk_floats, st));
    }
    {
      rwkv7_gemm_problem p = {w.h, Lw.w_fv, w.x, w.x1, M, C, 4 * C, 4 * C, 4 * C, C};
      int splits = 1;
      TRY(gemm_launch_ws(&p, 1, RWKV_EPI_RESID, w.splitk, w.splitk_floats, st, &splits));
      defer(splits, w.x1);
    }
  }
  if (b->n_logits) {
    TRY(launch_ln_rows(w.x, b->logit_rows, (const __half*)model->lnout_w,
                       (const __half*)model->lnout_b, w.lnout, b->n_logits, M, C, pend, st));
    if (b->logits) {
      rwkv7_gemm_problem p = {w.lnout, model->head, b->logits, nullptr, b->n_logits,
                              model->vocab, C, C, C, model->vocab};
      TRY(gemm_launch_ws(&p, 1, RWKV_EPI_STORE, w.splitk, w.splitk_floats, st));
    }
    if (b->next_ids) {
      // greedy head: per-row argmax folded into the GEMM epilogue, no logits stored
      if (cudaMemsetAsync(w.argmax_keys, 0, (size_t)b->n_logits * 8, st) != cudaSuccess)
        return rwkv_check_launch("argmax key memset");
      rwkv_chain_begin();  // the GEMM after the memset starts a plain-order chain
      rwkv7_gemm_problem p = {w.lnout, model->head, w.argmax_keys, nullptr, b->n_logits,
                              model->vocab, C, C, C, model->vocab};
      TRY(gemm_launch_ws(&p, 1, EPI_ARGMAX, nullptr, 0, st));
      TRY(launch_argmax_finish(w.argmax_keys, b->next_ids, b->n_logits, st));
    }
  }
  TRY(launch_scatter_state_x(w.xlast, (__half*)state->tmix_x, (__half*)state->cmix_x, b->slots, S,
                             L, ns, C, st));
  return RWKV_OK;
}
