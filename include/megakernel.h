/*
 * megakernel.h -- C ABI of libmegakernel (B200 / sm_100a persistent decode
 * megakernel for Qwen3-0.6B-shaped decoders).
 *
 * The first six functions are the drop-in surface of the reference's
 * `make lib` library (src/megakernel.cu:535-624, bound from Python in
 * host/bridge.py:39-67); their C signatures and meaning are unchanged.
 * Everything after them is an additive extension.
 *
 * Pointers named d_* are device pointers; all others are host pointers.
 * Status-returning extensions return MK_OK (0) or a negative MK_ERR_* code.
 */
#ifndef MEGAKERNEL_H_
#define MEGAKERNEL_H_

#ifdef __cplusplus
extern "C" {
#endif

enum {
  MK_OK = 0,
  MK_ERR_INVALID_ARG = -1, /* bad handle, pointer, token id or size */
  MK_ERR_CUDA = -2,        /* a CUDA runtime call failed */
  MK_ERR_TIMEOUT = -3,     /* a bounded in-kernel wait expired */
  MK_ERR_CAPACITY = -4,    /* position would exceed the KV capacity */
  MK_ERR_SHAPE = -5,       /* offsets match no compiled model shape */
  MK_ERR_LAUNCH = -6,      /* cooperative launch impossible (SMs busy, smem) */
  MK_ERR_OOM = -7          /* device allocation failed */
};

/* ---- reference surface (src/megakernel.cu:544-622) ---------------------- */

/* Replaces megakernel_init (src/megakernel.cu:544-585).  d_weights: device copy
 * of the flat binary (caller keeps it alive); offsets: 2 + 11*layers byte
 * offsets in host/bridge.py:89-96 order.  The model shape is inferred from
 * the offsets.  Returns NULL on failure (the reference never does). */
void* megakernel_init(void* d_weights, long long* offsets, int num_offsets);

/* Replaces megakernel_decode (src/megakernel.cu:588-591): feed one token at the
 * current position, return the greedy next token, advance the position.
 * Returns -1 on error (see megakernel_last_error). */
int megakernel_decode(void* handle, int input_token);

/* Replaces megakernel_reset (src/megakernel.cu:594-601): position 0, KV zeroed. */
void megakernel_reset(void* handle);

/* Replaces megakernel_get_pos (src/megakernel.cu:604-607). */
int megakernel_get_pos(void* handle);

/* Replaces megakernel_free (src/megakernel.cu:610-617). */
void megakernel_free(void* handle);

/* Replaces megakernel_sync (src/megakernel.cu:620-622): device synchronize. */
void megakernel_sync(void);

/* ---- extensions ----------------------------------------------------------- */

typedef struct mk_options {
  int device;            /* CUDA device ordinal; -1 = current device */
  int shape_id;          /* 0 d64, 1 d128, 2 tiny; -1 = infer from offsets */
  int max_seq;           /* KV capacity in positions; 0 = 8448 */
  int num_ctas;          /* persistent CTAs; 0 = one per SM */
  long long timeout_ns;  /* bound on every in-kernel wait; 0 = 1 s */
  int debug_skip_cta;    /* fault-injection hook for tests; -1 = off */
} mk_options;

/* Fill *opts with the defaults above. */
void megakernel_default_options(mk_options* opts);

/* megakernel_init with options and a status code. */
int megakernel_init_ex(void* d_weights, const long long* offsets, int num_offsets,
                       const mk_options* opts, void** out_handle);

/* Run n_steps decode steps in ONE kernel launch.  Step s feeds d_tokens[s] for
 * s < n_forced (teacher forcing / prefill) and the previous step's argmax
 * afterwards.  d_out[s] receives the argmax of step s.  d_logits, if not NULL,
 * receives [n_steps, vocab] fp32 logits.  stream: cudaStream_t, or NULL for the
 * default stream.
 * Blocks until the launch finishes; the position advances by n_steps. */
int megakernel_decode_n(void* handle, const int* d_tokens, int n_forced, int n_steps,
                        int* d_out, float* d_logits, void* stream);

/* Host-buffer convenience over decode_n: feeds the n_prompt prompt ids, then
 * generates n_gen tokens greedily (n_prompt + n_gen - 1 steps, one launch)
 * into out[n_gen].  Copies inputs in and results out itself. */
int megakernel_generate(void* handle, const int* prompt, int n_prompt, int n_gen, int* out);

/* Capture the fp32 logits of every megakernel_decode call (off by default);
 * megakernel_get_logits copies the latest ones to out[vocab]. */
int megakernel_set_logits_capture(void* handle, int enable);
int megakernel_get_logits(void* handle, float* out);

/* Position control and KV access (KV layout [layers, 2, kv_heads, max_seq,
 * head_dim] bf16, as src/kv_cache.cuh:9-32).  set_pos lets a caller inject
 * a prefilled cache. */
int megakernel_set_pos(void* handle, int pos);
void* megakernel_kv_ptr(void* handle);
long long megakernel_kv_bytes(void* handle);
int megakernel_max_seq(void* handle);
int megakernel_shape_id(void* handle);
int megakernel_num_ctas(void* handle);

/* Attention-merge kernel choice for later launches: 0 (default) picks the
 * two-level merge once a launch goes past 5 split-KV chunks per head
 * (positions > 640) and the direct merge before; 1 always
 * the direct merge; 2 always the kernel instance that carries the two-level
 * merge (it still merges directly below 5 chunks).  Results agree within
 * fp32 rounding; the choice only changes speed.  No reference counterpart. */
int megakernel_set_merge_mode(void* handle, int mode);

/* Last error of this handle (MK_OK if none) and a description of a code. */
int megakernel_last_error(void* handle);
const char* megakernel_error_string(int code);

/* Phase tracing: while set, every launch writes %globaltimer stamps (ns) for
 * its first `steps` steps into d_buf[steps][num_ctas][trace_points] (u64,
 * caller-owned device memory).  Points per layer l (index 7l + k): k=0 the
 * CTA's copy engine reaches layer l, 1 layer input ready, 2 q/k/v published,
 * 3 attention merged, 4 x after attention published, 5 MLP hidden published,
 * 6 layer output published; then 7L lm-head start, 7L+1 lm partial published,
 * 7L+2 next token known, 7L+3 ns spent waiting on activation hops (thread 0),
 * 7L+4 SM clock cycles over the step.  steps = 0 turns tracing off.
 * Profiling builds only (-DMK_TRACE_POINTS=1): the stamps are kernel code,
 * and this kernel is bound by its instruction-cache footprint; a default
 * build returns MK_ERR_INVALID_ARG for steps > 0. */
int megakernel_set_trace(void* handle, void* d_buf, int steps);
int megakernel_trace_points(void* handle);
/* Profiling aid: sub-phase stamps of layer 1 into d_buf[steps][num_ctas][64]
 * (needs megakernel_set_trace active; NULL turns it off).  Only in a library
 * built with -DMK_DETAIL_STAMPS=1; otherwise a non-NULL d_buf returns
 * MK_ERR_INVALID_ARG. */
int megakernel_set_trace_detail(void* handle, void* d_buf);

/* ---- decode without device allocation ------------------------------------ */

#define MK_NOALLOC_MAX_POS 2048           /* pos + n_steps must not exceed this */
#define MK_NOALLOC_SCRATCH_BYTES 932608   /* static device scratch per GPU */

/* No counterpart in the reference.  For callers that cannot allocate device
 * memory (a runtime that owns all device allocations, an allocator-free
 * loader, a plugin that must keep its footprint fixed): runs n_steps decode
 * steps of the graded shape (head_dim 64, intermediate 2816) like
 * megakernel_decode_n, but on caller-owned buffers only -- weights + offsets
 * as for megakernel_init, the KV cache d_kv ([layers, 2, kv_heads,
 * kv_max_seq, head_dim] bf16) starting at position pos, tokens in/out and
 * optional logits -- and calls no cudaMalloc/cudaFree.  Its scratch is a
 * fixed MK_NOALLOC_SCRATCH_BYTES array in the library's device image, held
 * on every GPU that loads the library until exit.  pos + n_steps beyond
 * MK_NOALLOC_MAX_POS or kv_max_seq returns MK_ERR_CAPACITY.  The first call
 * on a device (the current one) sets that device up with blocking copies:
 * make it before any stream capture.  All calls share the scratch, so calls
 * that overlap on the GPU race.  Blocks until done; returns MK_OK or an
 * MK_ERR_* code.  The caller tracks the position (pos += n_steps).
 * d_weights and d_kv must be 16-byte aligned (MK_ERR_INVALID_ARG otherwise);
 * a forced token id outside the vocabulary returns MK_ERR_INVALID_ARG.  Like
 * megakernel_decode_n it runs the kernel instance with the two-level
 * attention merge once pos + n_steps - 1 goes past 5 chunks per head (> 640). */
int megakernel_decode_noalloc(const void* d_weights, const long long* offsets, int num_offsets,
                              void* d_kv, int kv_max_seq, int pos, const int* d_tokens,
                              int n_forced, int n_steps, int* d_out, float* d_logits,
                              void* stream);

/* ---- batched path building blocks (no reference counterpart) -------------- */

/* One tcgen05 GEMM as the batched decode uses it: d_out[r][n] =
 * sum_k d_x[r][k] * d_w[n][k] for r < rows (<= 64), with d_x fp32 [rows x K]
 * and d_w bf16 [N x K] row-major (K, N multiples of 64).  x enters the
 * tensor cores as two bf16 terms (hi, lo).  Allocates scratch; synchronous.
 * Returns MK_OK or an MK_ERR_* code. */
int megakernel_tc_gemm_test(const float* d_x, int rows, const void* d_w, int K, int N, float* d_out,
                            void* stream);
/* The same with K split over `ksplit` (1..4) CTAs per 64-column output tile:
 * the CTAs of a tile form a thread-block cluster, ranks 1..ksplit-1 push
 * their partial tiles into rank 0's shared memory and rank 0 sums them (the
 * split-K path of the batched O and down projections).  Every split must keep at least one
 * 64-column K block (MK_ERR_INVALID_ARG otherwise). */
int megakernel_tc_gemm_test_split(const float* d_x, int rows, const void* d_w, int K, int N, int ksplit,
                                  float* d_out, void* stream);
/* The same on e4m3 weights: d_w8 [N][K] e4m3 bytes with per-row scales
 * d_scale[N] (W = scale * e4m3), through the GEMM's e4m3 -> bf16 converter
 * warps (the path megakernel_batch_init_ex(..., MK_W_FP8_E4M3) runs). */
int megakernel_tc_gemm_test_e4m3(const float* d_x, int rows, const void* d_w8, const float* d_scale, int K, int N,
                                 float* d_out, void* stream);

/* Parallel prefill (no reference counterpart; replaces the token-serial
 * prompt loop of host/bridge.py:158-162): feeds d_tokens[n_tokens] (device)
 * at positions pos .. pos+n-1 of this engine's cache, 64 positions per
 * batched tcgen05 step, advances pos by n and writes the greedy token after
 * the last prompt token to d_next (device).  Graded (head_dim 64) shape
 * only (MK_ERR_SHAPE otherwise); synchronous.  megakernel_generate uses it
 * for that shape (set MK_SERIAL_PREFILL to force the token-serial loop). */
int megakernel_prefill(void* handle, const int* d_tokens, int n_tokens, int* d_next, void* stream);

/* ---- batched decode (no reference counterpart) ----------------------------
 * Up to 64 sequences advance together, one token each per step, each at its
 * own position; matrix products run on tcgen05 tensor cores with the
 * sequences as the M dimension.  Same flat weights + offsets as
 * megakernel_init (d64 shape only).  KV layout: [batch][L][2][KVH][max_seq][hd]
 * bf16, i.e. one reference-layout cache (src/kv_cache.cuh:9-32) per sequence.
 * Positions start at 0; every step advances every sequence by one. */
void* megakernel_batch_init(const void* d_weights, const long long* offsets, int num_offsets, int batch,
                            int max_seq);
/* As megakernel_batch_init with storage options (no reference counterpart),
 * `flags` a combination of:
 *   MK_KV_FP8_E4M3  the KV cache in e4m3 -- the same [batch][L][2][KVH]
 *                   [max_seq][head_dim] layout in bytes (half the cache;
 *                   K/V rounded to nearest, saturating; attention then runs
 *                   in f16 on the tensor cores);
 *   MK_W_FP8_E4M3   the GEMMs on an e4m3 copy of the weights made at init
 *                   (one scale per row, max |w| / 448; half the weight
 *                   bytes; the caller's bf16 weights stay in use for the
 *                   embedding and the norms).
 * MK_KV_BF16 (0) is the reference's precision.  NULL on failure. */
enum { MK_KV_BF16 = 0, MK_KV_FP8_E4M3 = 1, MK_W_FP8_E4M3 = 2 };
void* megakernel_batch_init_ex(const void* d_weights, const long long* offsets, int num_offsets, int batch,
                               int max_seq, int flags);
void megakernel_batch_free(void* handle);
int megakernel_batch_size(void* handle);
/* One step: d_tokens[batch] (device) -> d_out[batch] next greedy tokens;
 * d_logits (device, [batch][vocab] fp32) may be NULL.  Synchronous. */
int megakernel_batch_step(void* handle, const int* d_tokens, int* d_out, float* d_logits, void* stream);
/* n_steps steps: step t < n_forced consumes d_forced[t][batch], later steps
 * consume the previous step's outputs; d_out[n_steps][batch].  Synchronous. */
int megakernel_batch_decode_n(void* handle, const int* d_forced, int n_forced, int n_steps, int* d_out,
                              void* stream);
int megakernel_batch_set_pos(void* handle, const int* h_pos);   /* h_pos[batch] */
int megakernel_batch_get_pos(void* handle, int* h_pos);
void* megakernel_batch_kv_ptr(void* handle);
long long megakernel_batch_kv_bytes(void* handle);
int megakernel_batch_last_error(void* handle);

/* ---- tensor parallelism over NVLink (no reference counterpart) ------------
 * configs[4](b): one process per GPU, tp_size in {2, 4, 8} (graded d64
 * shape; the tiny test shape also at 2).  Each rank reads its slice of the
 * MLP (gate/up rows and down columns [rank I/tp, (rank+1) I/tp)) and of the
 * LM head (vocab rows [rank V/tp, (rank+1) V/tp)); attention, QKV and O stay
 * replicated.  Inside the kernel each rank stores its partial down projection
 * (1024 fp32 per layer) and its per-CTA (max, index) pairs straight into
 * every rank's exchange buffer over NVLink; every rank sums the partials in
 * rank order, so all ranks hold identical activations and pick the same
 * token.  Set-up: megakernel_tp_init on every rank, exchange the 64-byte
 * handles of megakernel_tp_ipc_handle (rank order), then
 * megakernel_tp_connect.  After that every decode call of this ABI
 * (megakernel_decode, _decode_n, _generate, _prefill, _set_pos, _reset) works
 * in TP mode, and all ranks must make the same calls with the same arguments.
 * Captured logits hold only this rank's vocab rows. */
int megakernel_tp_init(void* d_weights, const long long* offsets, int num_offsets,
                       const mk_options* opts, int tp_rank, int tp_size, void** out_handle);
int megakernel_tp_ipc_handle(void* handle, void* out_64_bytes);
int megakernel_tp_connect(void* handle, const void* handles_tp_size_x_64_bytes);
int megakernel_tp_info(void* handle, int* rank, int* size);
/* Check hook for the in-kernel exchange (no reference counterpart): copies
 * the payloads of this GPU's tensor-parallel exchange slots of the last
 * layer of the last step -- every rank's partial down projection as it
 * arrived here over NVLink (own slot written locally) -- into d_out
 * [tp_size][hidden] fp32 on the engine's device.  Synchronous. */
int megakernel_tp_exchange_slots(void* handle, float* d_out);

/* ---- host-only helpers (no GPU needed) ----------------------------------- */

/* Shape id matching a flat-binary offsets array, or MK_ERR_SHAPE. */
int megakernel_infer_shape(const long long* offsets, int num_offsets);

/* fp32 RoPE tables [positions, head_dim/2] exactly as the kernel uses them. */
int megakernel_rope_table(int head_dim, double theta, int positions, float* cos_out,
                          float* sin_out);

/* Bytes each CTA streams through its shared-memory ring for one step at
 * position pos (weights + cached K/V): bytes_per_cta[num_ctas]. */
int megakernel_plan_bytes(int shape_id, int num_ctas, int pos, long long* bytes_per_cta);

#ifdef __cplusplus
}
#endif

#endif /* MEGAKERNEL_H_ */
