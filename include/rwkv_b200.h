/*
 * rwkv_b200.h -- C ABI of the B200 (sm_100a) RWKV-7 forward hot path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream, allocates no
 * device memory itself (scratch comes from a caller-provided workspace), and
 * returns 0 on success or a nonzero RWKV_ERR_* code; the message is available
 * from rwkv_b200_last_error() (thread-local). There is no CPU fallback.
 *
 * Tensor conventions: fp16 activations and weights ("half" = IEEE binary16,
 * passed as void*), fp32 wkv state, row-major. Weight matrices keep the
 * checkpoint's [out, in] orientation so both the GEMV (decode) and the
 * K-major tensor-core GEMM (prefill) read them contiguously along `in`.
 *
 * Reference interfaces replaced (yuyi2439/rwkv-tl, paths within that project):
 *   rwkv7_dplr_step     <- Kernels.fused_dplr      src/rwkv_tl/kernels/dplr.py:256-270
 *                          (torch.ops.rwkv_tl.fused_dplr, src/rwkv_tl/operators/__init__.py:315-322)
 *   rwkv7_dplr_seq      <- Kernels.fused_dplr_T    src/rwkv_tl/kernels/dplr.py:272-285
 *   rwkv7_dplr_chunked  <- Kernels.fused_dplr_T (chunk-parallel, batched over sequences)
 *   rwkv7_gemm_f16      <- Kernels.fused_rkv_gemm / ffn_h / ffn_v / out_mm
 *                          src/rwkv_tl/kernels/gemm.py:215-305
 *   rwkv7_forward       <- RWKV7Base.prefill / RWKV7Base.decode layer loops
 *                          demo/_rwkv7_base.py:74-98 (TMIX :153-206 / :223-272,
 *                          CMIX :285-290 / :300-308), batched over sequences
 *   rwkv7_decode_gemv   <- RWKV7Base.decode (demo/_rwkv7_base.py:74-87) for
 *                          small batches, the CUDA-Graph decode body of
 *                          demo/cuda_graph.py:111-128
 */
#ifndef RWKV_B200_H_
#define RWKV_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RWKV_B200_ABI_VERSION 2

enum {
  RWKV_OK = 0,
  RWKV_ERR_ARG = 1,     /* bad shape / null pointer / unsupported size */
  RWKV_ERR_CUDA = 2,    /* a CUDA launch or runtime call failed */
  RWKV_ERR_SPACE = 3    /* workspace too small */
};

/* Rounding semantics. The reference's fp16 decode path rounds to fp16 only at
 * its fused-kernel stores (src/rwkv_tl/kernels/{lerp,gates,dplr}.py); its
 * prefill path rounds after every torch op (demo/_rwkv7_base.py:223-310).
 * RWKV_SEM_DECODE reproduces the former, RWKV_SEM_PREFILL the latter. */
enum { RWKV_SEM_DECODE = 0, RWKV_SEM_PREFILL = 1 };

/* GEMM epilogues: C = f(A @ B^T) with fp32 accumulation. */
enum {
  RWKV_EPI_STORE = 0,  /* C = fp16(acc)                                  */
  RWKV_EPI_RESID = 1,  /* C = fp16(R + fp16(acc))          (x0 + y @ W)  */
  RWKV_EPI_RELUSQ = 2, /* C = fp16(relu(fp16(acc))^2)      (FFN key)     */
  RWKV_EPI_STORE_F32 = 3, /* C = acc as fp32 (C is float*, ldc in floats)   */
  RWKV_EPI_LORA_ACT = 4,  /* LoRA-down of a 4-problem group v, w, a, g: C =
                             fp16(act(fp16(acc))), act = tanh for problem 1
                             (w), sigmoid for problem 3 (g), identity else  */
  RWKV_EPI_LORA_ACT2 = 5  /* as LORA_ACT, and the fp16 remainder act - hi of
                             problems 1 / 3 is written 64 / 128 columns to the
                             right, so hi + lo carries the fp32 activation   */
};

/* Per-layer weights (device pointers, fp16). C = n_embd, H = C/64. */
typedef struct rwkv7_layer {
  const void* ln1_w; const void* ln1_b;   /* [C]                                 */
  const void* ln2_w; const void* ln2_b;   /* [C]                                 */
  const void* mix6;       /* [6, C]  x_r, x_w, x_k, x_v, x_a, x_g                  */
  const void* w_rkv;      /* [3C, C] receptance | key | value weights ([out, in])  */
  const void* w_lora_dn;  /* [288, C] v1^T(32) | w1^T(64) | a1^T(64) | g1^T(128)   */
  const void* w_lora_up;  /* [288, C] v2(32) | w2(64) | a2(64) | g2(128)  ([r, C]) */
  const void* w0; const void* a0; const void* v0;   /* [C] gate biases           */
  const void* k_k; const void* k_a;       /* [C]                                 */
  const void* r_k;        /* [C] (= [H, 64])                                       */
  const void* lnx_w; const void* lnx_b;   /* [C] per-head GroupNorm affine       */
  const void* w_o;        /* [C, C] output projection ([out, in])                  */
  const void* ffn_x_k;    /* [C]                                                   */
  const void* w_fk;       /* [4C, C] FFN key                                       */
  const void* w_fv;       /* [C, 4C] FFN value                                     */
  const void* w_lora_up_t; /* [C, 512] K-major LoRA up for the tensor-core path:
                              v2^T | 0 (32 each) | w2^T | w2^T | a2^T | g2^T | g2^T */
} rwkv7_layer;

typedef struct rwkv7_model {
  int n_layer, n_embd, vocab;
  int rank_v, rank_w, rank_a, rank_g;     /* must be 32, 64, 64, 128          */
  const void* emb;        /* [V, C] embedding with LN0 already applied           */
  const void* head;       /* [V, C]                                              */
  const void* lnout_w; const void* lnout_b; /* [C]                               */
  const rwkv7_layer* layers;  /* HOST array of n_layer entries                  */
} rwkv7_model;

/* Recurrent state of `n_slots` sequences, one contiguous block per tensor:
 *   rnn    fp32 [L, n_slots, H, 64, 64]   (row = value index, column = key index,
 *                                          the layout of State.tmix[i]["rnn"])
 *   tmix_x fp16 [L, n_slots, C]           (State.tmix[i]["x"])
 *   cmix_x fp16 [L, n_slots, C]           (State.cmix[i]["x"])
 * (src/rwkv_tl/state.py:31-44, with a leading layer and slot dimension). */
typedef struct rwkv7_state {
  void* rnn; void* tmix_x; void* cmix_x;
  int n_slots;
} rwkv7_state;

/* A batch of token rows. Rows of sequence s are [cu_seqlens[s], cu_seqlens[s+1]),
 * consecutive in time; sequence s uses state slot slots[s] (NULL: slot s).
 * All arrays are device pointers. */
typedef struct rwkv7_batch {
  int n_rows, n_seqs;
  const int64_t* tokens;    /* [n_rows]                                         */
  const int* cu_seqlens;    /* [n_seqs + 1]                                     */
  const int* row_seq;       /* [n_rows] sequence index of each row              */
  const int* slots;         /* [n_seqs] or NULL                                 */
  int n_logits;             /* rows that produce logits (0: state update only)  */
  const int* logit_rows;    /* [n_logits] row indices                           */
  void* logits;             /* fp16 [n_logits, V], or NULL                      */
  int semantics;            /* RWKV_SEM_DECODE or RWKV_SEM_PREFILL              */
  int64_t* next_ids;        /* [n_logits] greedy next token of each logit row,
                               or NULL. The head GEMM then reduces each row to
                               its argmax (lowest id among equal fp16 logits,
                               like torch.argmax) in its epilogue: no logits are
                               stored unless `logits` is also given. At least
                               one of logits / next_ids when n_logits > 0.
                               Replaces head @ x followed by the sampler's argmax
                               (demo/_rwkv7_base.py:86-87, demo/sampling.py:13-70) */
} rwkv7_batch;

const char* rwkv_b200_last_error(void);
int rwkv_b200_abi_version(void);
/* Number of kernel launches this library has issued from the host so far (a
 * captured CUDA graph replays its kernels without passing through here). */
unsigned long long rwkv_b200_launch_count(void);
/* Nonzero if, since the last call, a kernel on the current device gave up on a
 * bounded wait instead of spinning forever (bit 0 a GEMM pipeline barrier, bit 1 a
 * grid barrier of the persistent decode kernel), or a chunked-wkv kernel found a
 * sequence table out of range and skipped that sequence, or its scan gave up on a
 * bounded wait for a chunk record (bit 2). Reading clears it.
 * Synchronous (reads device memory). */
int rwkv_b200_device_error(void);
/* Makes one of the library's bounded device waits run out on purpose, to show that
 * failure detection fires and the context stays usable: which = 0 the GEMM pipeline's
 * mbarrier wait (sets bit 0 of rwkv_b200_device_error, ~1 s), 1 the persistent decode
 * kernel's grid-barrier and mbarrier waits (bit 1, ~0.4 s), 2 the chunk scan's record
 * wait (bit 2, ~0.2 s). Each launches one small kernel that runs the same wait
 * function on a barrier nothing signals; it writes an int at scratch + 16 (nonzero:
 * the wait gave up). scratch: 32 zeroed, 16-byte aligned device bytes. No GPU fault,
 * trap or hang is involved. No counterpart in the reference (it has no device waits). */
int rwkv_b200_wait_selftest(int which, void* scratch, void* stream);

/* wkv7 DPLR step, batched over n_seq independent sequences (T = 1):
 *   sa[v] = sum_j S[v,j] a[j];  S[v,k] = S[v,k] w[k] + sa[v] b[k] + v[v] k[k];
 *   y[v]  = sum_k S[v,k] r[k]      (S updated in place, y stored fp16)
 * S: fp32 [n_seq, H, 64, 64]; r, w, k, v, a, b, y: fp16 [n_seq, H, 64].
 * Argument order follows fused_dplr(S, R, W, K, V, A, B). */
int rwkv7_dplr_step(void* S, const void* r, const void* w, const void* k, const void* v,
                    const void* a, const void* b, void* y, int n_seq, int H, void* stream);

/* One decode token of n_seq sequences through the whole per-head attention tail:
 * the wkv7 step above on state S[slots[i]] (slots NULL: i), then per-head GroupNorm
 * (eps 64e-5, affine lnx_w/lnx_b), the bonus (sum_j r*k*r_k) * v and the g gate:
 *   out = (GN(y) + bonus) * g      (fp16 rounding points of `semantics`)
 * r, w, k, v, a, b, g, out: fp16 [n_seq, H*64]; r_k, lnx_w, lnx_b: fp16 [H*64];
 * S: fp32 [slots, H, 64, 64]. Replaces fused_dplr + fused_gn_rkrk and the g
 * multiply of the decode TMIX (src/rwkv_tl/kernels/dplr.py:237-270,
 * demo/_rwkv7_base.py:202-206). */
int rwkv7_wkv_gn_step(void* S, const int* slots, const void* r, const void* w, const void* k,
                      const void* v, const void* a, const void* b, const void* g,
                      const void* r_k, const void* lnx_w, const void* lnx_b, void* out,
                      int n_seq, int H, int semantics, void* stream);

/* The same recurrence over T consecutive tokens of one sequence (fused_dplr_T):
 * r..b, y: fp16 [T, H, 64]; S: fp32 [H, 64, 64] updated in place. */
int rwkv7_dplr_seq(void* S, const void* r, const void* w, const void* k, const void* v,
                   const void* a, const void* b, void* y, int T, int H, void* stream);

/* Chunk-parallel form of the same recurrence for n_seq sequences of T tokens
 * (replaces fused_dplr_T's serial loop for long T):
 * r..b, y: fp16 [n_seq, T, H, 64]; S: fp32 [n_seq, H, 64, 64] updated in place.
 * Needs rwkv7_dplr_chunked_workspace_bytes(n_seq, T, H) bytes of scratch. */
size_t rwkv7_dplr_chunked_workspace_bytes(int n_seq, int T, int H);
int rwkv7_dplr_chunked(void* S, const void* r, const void* w, const void* k, const void* v,
                       const void* a, const void* b, void* y, int n_seq, int T, int H,
                       void* workspace, size_t workspace_bytes, void* stream);

/* rwkv7_dplr_chunked for callers that cannot allocate device memory (a frozen
 * memory pool, a host framework that only hands out input/output buffers):
 * no workspace argument, no allocation. Its scratch is a fixed 32 MiB device
 * array inside this library, so it accepts only problems whose
 * rwkv7_dplr_chunked_workspace_bytes(n_seq, T, H) is at most 32 MiB and
 * returns RWKV_ERR_SPACE otherwise. The first call on a device looks up the
 * array's address (do it before any stream capture). All calls share the one
 * array: calls that overlap on the GPU (different streams) race. The looked-up
 * address is cached per device; after cudaDeviceReset in the same process it is
 * stale, so do not call this again after a reset. No counterpart in the reference. */
int rwkv7_dplr_chunked_noalloc(void* S, const void* r, const void* w, const void* k,
                               const void* v, const void* a, const void* b, void* y, int n_seq,
                               int T, int H, void* stream);

/* Token sampling, one kernel for B rows of fp16 logits [B, V] (V <= 65536, a multiple
 * of 8, logits 16-byte aligned): repetition penalty on each row's seen ids (CSR:
 * seen[seen_cu[b] .. seen_cu[b+1]); NULL for none), then greedy argmax (lowest id on
 * ties) when temperature <= 0; else logits / temperature, top-k (0 = off; ties with
 * the k-th logit kept), nucleus top-p (1 = off; a token is kept when the mass ranked
 * above it is <= top_p) and one draw per row from the kept softmax at the caller's
 * uniform uniforms[b] in [0, 1). out: int64 [B]. Replaces sample_logits
 * (demo/sampling.py:13-70): same rules, same distribution; ids differ from
 * torch.multinomial's for the same seed. Bit-reproducible for fixed inputs. */
int rwkv7_sample(const void* logits, int B, int V, float temperature, int top_k, float top_p,
                 float repetition_penalty, const int64_t* seen, const int* seen_cu,
                 const float* uniforms, int64_t* out, void* stream);

/* Grouped fp16 GEMM, up to 4 independent problems in one launch:
 *   C_g[M_g, N_g] = epi( A_g[M_g, K_g] @ B_g[N_g, K_g]^T )
 * A row-major (lda), B row-major [N, K] (ldb), C/R row-major (ldc). K_g must be
 * a multiple of 32, lda/ldb/ldc multiples of 8; M and N arbitrary. */
typedef struct rwkv7_gemm_problem {
  const void* A; const void* B; void* C; const void* R;
  int M, N, K, lda, ldb, ldc;
} rwkv7_gemm_problem;
int rwkv7_gemm_f16(const rwkv7_gemm_problem* problems, int n_problems, int epilogue,
                   void* stream);

/* Full forward of a token batch through all layers (prefill of any number of
 * sequences, or one decode step of many sequences), updating `state` in place
 * and writing logits for batch->logit_rows. Needs a device workspace of at
 * least rwkv7_forward_workspace_bytes(...) bytes (256-byte aligned). */
size_t rwkv7_forward_workspace_bytes(const rwkv7_model* model, int n_rows, int n_seqs,
                                     int n_logits);
int rwkv7_forward(const rwkv7_model* model, const rwkv7_batch* batch,
                  const rwkv7_state* state, void* workspace, size_t workspace_bytes,
                  void* stream);

/* One decode step of n_seqs (1..8) sequences, one token each, through the
 * small-batch path. n_seqs <= 4 (two sequences per launch): one persistent
 * cooperative kernel per launch, one CTA per SM, grid barriers between the
 * three phases of each layer, weight slices staged into shared memory by TMA
 * one phase ahead, GEMVs on the tensor cores. n_seqs 5..8 (or when the device
 * or pointer alignment does not allow the persistent kernel): three fused
 * kernels per layer (LN+mix+r/k/v/LoRA-down GEMV; per-head gates+wkv+GroupNorm+
 * output projection; LN2+FFN) and the head GEMV, chained with programmatic
 * dependent launch. Decode rounding semantics.
 * tokens: device int64 [n_seqs]; slots: device int [n_seqs] or NULL; logits:
 * fp16 [n_seqs, V]. n_embd must be 768 or 1024. Same result as
 * rwkv7_forward with RWKV_SEM_DECODE on one token per sequence. */
size_t rwkv7_decode_gemv_workspace_bytes(const rwkv7_model* model, int n_seqs);
int rwkv7_decode_gemv(const rwkv7_model* model, const int64_t* tokens, int n_seqs,
                      const int* slots, const rwkv7_state* state, void* logits, void* workspace,
                      size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* RWKV_B200_H_ */
