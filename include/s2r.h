/*
 * s2r.h — C ABI of the B200 decode engine for SheetSage2-Refined's
 * grammar-constrained greedy decoder token loop.
 *
 * The engine replaces the reference's `BatchDecoder`
 * (sheetsage2_refined/engine.py:52-369): a batch of independent decode
 * slots, each with its own paged self-attention K/V cache, resident
 * cross-attention K/V of its encoder window, grammar state and output
 * buffer.  One step feeds every live slot its last token through the
 * post-LayerNorm decoder (decoder.py:58-151), picks the next token under the
 * grammar mask with a greedy argmax and advances the grammar, all on the GPU.
 *
 * Conventions
 *  - Every entry point returns an `s2r_status`; none aborts.  The message of
 *    the last failure on the calling thread is `s2r_last_error()`.
 *  - Pointers to caller data may be host or device memory (unified
 *    addressing) unless stated otherwise; the engine copies what it keeps.
 *  - `stream` is a `cudaStream_t` (NULL: the legacy default stream).  Work is
 *    ordered on it; entry points that return host data synchronise it.
 *  - Not thread-safe: one host thread drives one engine (as the reference).
 */
#ifndef S2R_H
#define S2R_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define S2R_ABI_VERSION 1
#define S2R_PAGE_TOKENS 64 /* tokens per self-attention K/V page */
#define S2R_NO_TARGET INT64_MAX

typedef enum s2r_status {
  S2R_OK = 0,
  S2R_EINVAL = 1,   /* bad argument (the reference raises ValueError/IndexError) */
  S2R_ECUDA = 2,    /* a CUDA call failed */
  S2R_ENOMEM = 3,   /* device memory or K/V pages exhausted */
  S2R_ESTATE = 4,   /* call out of order (e.g. take of a slot that is not loaded) */
  S2R_ENOTSUP = 5,  /* shape the kernels do not support */
  S2R_EDEVICE = 6   /* a kernel found a broken invariant, reported it and skipped its work */
} s2r_status;

typedef enum s2r_grammar_kind {
  S2R_GRAMMAR_CLASS = 0, /* TokenGrammar: 13 token classes + per-slot state */
  S2R_GRAMMAR_TABLE = 1  /* synthetic [states, vocab] table grammar */
} s2r_grammar_kind;

typedef enum s2r_dtype { S2R_F32 = 0, S2R_BF16 = 1 } s2r_dtype;

/* Decoder shape and engine sizes.
 * Replaces DecoderConfig (decoder.py:12-21) plus the BatchDecoder constructor
 * arguments `batch` and `frames` (engine.py:55-66). */
typedef struct s2r_config {
  int32_t vocab_size;
  int32_t width;      /* multiple of 64, at most 4096 */
  int32_t layers;
  int32_t heads;      /* width / heads must be 64 */
  int32_t ffn_width;  /* multiple of 64, at most 4096 */
  int32_t max_tokens; /* decoder context; position rows = max_tokens + 2 */
  int32_t batch;      /* decode slots */
  int32_t frames;     /* cross-attention frames held per slot */
  int32_t kv_pages;   /* self K/V pool in pages of S2R_PAGE_TOKENS tokens;
                         0 = batch * ceil(max_tokens / S2R_PAGE_TOKENS) */
  int32_t flags;      /* S2R_FLAG_* */
} s2r_config;

#define S2R_FLAG_NO_PDL 1u   /* launch without programmatic dependent launch */
#define S2R_FLAG_NO_GRAPH 2u /* issue steps as plain launches, no CUDA graph */
/* 4u, 8u, 16u: not flags (s2r_create rejects any bit but these three) */
#define S2R_FLAG_NO_TENSOR_CORE 32u /* every projection on the CUDA-core kernel (by default the cross K/V
                                       projection at load, prefill chunks of more than 8 rows, and
                                       with batch >= 16 the step projections run on tcgen05 tensor
                                       cores) */

/* One decoder layer's float32 parameters, named as in
 * TokenDecoder.state_dict() (decoder.py:28-84).  Linear weights are
 * [out, in] row-major, as torch stores them. */
typedef struct s2r_layer_weights {
  const float *self_q_w, *self_q_b, *self_k_w, *self_k_b;
  const float *self_v_w, *self_v_b, *self_out_w, *self_out_b;
  const float *self_norm_w, *self_norm_b;
  const float *cross_q_w, *cross_q_b, *cross_k_w, *cross_k_b;
  const float *cross_v_w, *cross_v_b, *cross_out_w, *cross_out_b;
  const float *cross_norm_w, *cross_norm_b;
  const float *fc1_w, *fc1_b, *fc2_w, *fc2_b;
  const float *final_norm_w, *final_norm_b;
} s2r_layer_weights;

/* Replaces the weight copies BatchDecoder makes at construction
 * (engine.py:118-123): Linear weights and biases and the tied output
 * embedding are rounded to bfloat16 on the device; embeddings used for the
 * lookup and LayerNorm parameters stay float32. */
typedef struct s2r_weights {
  const float* token_embedding;    /* [vocab_size, width] */
  const float* position_embedding; /* [max_tokens + 2, width] */
  const float* embedding_norm_w;   /* [width] */
  const float* embedding_norm_b;   /* [width] */
  const s2r_layer_weights* layers; /* [layers] (host array of structs) */
} s2r_weights;

/* Replaces TokenGrammar construction (grammar.py:79-97) or, for synthetic
 * vocabularies, a table grammar.  Arrays are host or device memory. */
typedef struct s2r_grammar {
  int32_t kind;                  /* s2r_grammar_kind */
  const int8_t* token_class;     /* CLASS: [vocab] class 0..12 of each token */
  const int32_t* field_of_class; /* CLASS: [13] (grammar.py:52) */
  const double* time_seconds;    /* [vocab] seconds of time tokens, -inf otherwise */
  int32_t states;                /* TABLE: number of states */
  int32_t multiplier;            /* TABLE: s' = (multiplier * s + token) mod states */
  const uint8_t* table;          /* TABLE: [states, vocab] 1 = allowed */
} s2r_grammar;

typedef struct s2r_ctx s2r_ctx;

/* ABI version of the loaded library (S2R_ABI_VERSION it was built with). */
int32_t s2r_abi_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* s2r_last_error(void);

/* Build an engine on `device`: allocate caches and state, copy and round the
 * weights, copy the grammar.  Every slot starts finished and unloaded.
 * Replaces BatchDecoder.__init__ (engine.py:55-149). */
int32_t s2r_create(const s2r_config* config, const s2r_weights* weights, const s2r_grammar* grammar,
                   int32_t device, s2r_ctx** out);

/* Free everything the engine owns.  Replaces dropping the engine
 * (transcribe.py:212 frees the old caches before a rebuild). */
int32_t s2r_destroy(s2r_ctx* ctx);

/* Additive float32 bias on the logits of every slot ([vocab], NULL clears),
 * applied after the bfloat16 logits are widened and before the grammar mask.
 * Replaces the `mode_bias` term (engine.py:77-80,316-317). */
int32_t s2r_set_logit_bias(s2r_ctx* ctx, const float* bias);

/* Frame-head rescoring terms, in the reference's FRAME_TERMS order
 * (engine.py:29-38): root, bass, detail, quality, key, key_boundary,
 * downbeat, meter. */
#define S2R_FRAME_TERMS 8

/* Frame-head rescoring configuration (engine.py:81-116): one weight per term
 * (0 disables the term), the vocabulary spans [start, end) it moves, the
 * meter tables and the vocabulary's time resolution.  Host pointers. */
typedef struct s2r_rescore {
  float weight[S2R_FRAME_TERMS];
  int32_t bass_span[2];    /* chord_bass block */
  int32_t detail_span[2];  /* chord_detail start, start + NO_CHORD */
  int32_t key_span[2];     /* key block */
  int32_t eighth_span[2];  /* eighth_position block */
  int32_t meter_span[2];   /* meter block */
  const int32_t* meter_beats; /* [meter block size] min(numerator, 16) - 1 of each meter */
  const int32_t* meter_unit;  /* [meter block size] denominator of each meter */
  int32_t time_hz;            /* time tokens per second of the vocabulary */
} s2r_rescore;

/* Enable frame-head rescoring with `rs` (NULL or all-zero weights: off).
 * Needs the class grammar.  Allocates the per-slot frame tables (float32
 * [batch][frames][width]: 12 root, 12 bass, NO_CHORD detail, NO_CHORD
 * quality, 24 key, 1 key_boundary, 1 downbeat, 16 meter).  Synchronises the
 * device.  Replaces the `frame_weight` argument of BatchDecoder
 * (engine.py:81-116); the terms are added to the logits as engine.py:318-347
 * does and the state they read advances as engine.py:358-369 does. */
int32_t s2r_set_rescore(s2r_ctx* ctx, const s2r_rescore* rs);

/* The window's per-frame tables of `slot` for frame-head rescoring
 * (engine.py:218-224): tables[t] holds rows[t] rows of the term's width
 * (float32, host or device; NULL or 0 rows: the term's table is zero); rows
 * beyond the engine's frames are ignored.  Call before s2r_load_slot of the
 * same window.  Replaces the `frame_logp` argument of BatchDecoder.load. */
int32_t s2r_load_frame_tables(s2r_ctx* ctx, int32_t slot, const float* const* tables, const int32_t* rows,
                              void* stream);

/* Start `slot` on a window.  `memory` is the encoder memory
 * [memory_frames, width] (float32 or bfloat16); cross-attention sees its
 * first `frames` frames (1 <= frames <= min(memory_frames, config.frames)).
 * `prefix` (host, n_prefix >= 1 tokens, containing OUT = 3) is prefilled: the
 * K/V of prefix[0 .. n-2] are written, the grammar state is replayed from the
 * token after OUT, and the slot resumes with token prefix[n-1] at position
 * n-1 (n_prefix <= max_tokens - 1).  `stop_seconds` ends the slot at the
 * first time token at or after it (+inf: never).  `target` is the table
 * grammar's generated-token count (S2R_NO_TARGET: none).
 * The cross K/V of every layer is projected in one tensor-core launch; the
 * prefix is prefilled in chunks of 128 positions, chunks of more than 8 on
 * tensor cores (the arithmetic of the reference's own prefill, so equal to
 * forcing the prefix token by token within the parity tolerance), shorter
 * ones on the decode step's kernels (equal bit for bit).
 * Replaces BatchDecoder.load (engine.py:180-232) without rescoring tables. */
int32_t s2r_load_slot(s2r_ctx* ctx, int32_t slot, const void* memory, int32_t memory_dtype,
                      int32_t memory_frames, int32_t frames, const int64_t* prefix, int32_t n_prefix,
                      double stop_seconds, int64_t target, void* stream);

/* Advance every slot by `n_steps` tokens; finished slots stay put.  No host
 * synchronisation.  Replaces BatchDecoder.run (engine.py:234-246). */
int32_t s2r_step(s2r_ctx* ctx, int32_t n_steps, void* stream);

/* One step with test hooks (host arrays, each may be NULL): `forced[slot]` >=
 * 0 commits that token instead of the greedy choice (teacher forcing);
 * `logits` receives the raw float32 logits [batch, vocab] (bfloat16-rounded,
 * before bias and mask); `greedy` receives the masked argmax of every slot.
 * Synchronises `stream`.  No counterpart in the reference's engine; its
 * teacher-forced logits come from TokenDecoder.forward (decoder.py:118-124). */
int32_t s2r_step_debug(s2r_ctx* ctx, const int64_t* forced, float* logits, int64_t* greedy, void* stream);

/* Copy the per-slot finished flags to host `finished` [batch] (synchronises).
 * Returns S2R_EDEVICE if a kernel has reported an error since the last check.
 * Replaces the device read of BatchDecoder.finished (engine.py:248-252). */
int32_t s2r_poll_finished(s2r_ctx* ctx, uint8_t* finished, void* stream);

/* Copy slot's tokens out[0 .. position] to host `tokens`, append EOS when the
 * last token is not EOS, report the end reason (0 running, 1 eos, 2 stop,
 * 3 limit) and release the slot's K/V pages.  Fails with S2R_EINVAL if
 * `capacity` is too small (`*length` then holds the size needed).
 * Replaces BatchDecoder.take (engine.py:254-262). */
int32_t s2r_take(s2r_ctx* ctx, int32_t slot, int64_t* tokens, int32_t capacity, int32_t* length,
                 int32_t* ended, void* stream);

/* Asynchronous poll: enqueue on `stream`, behind the work already there, a
 * copy of every slot's finished flag (and of the device error word) to host
 * memory the engine owns, and return at once.  The host can queue more steps
 * before it reads the flags with s2r_poll_finished_ready, so the GPU keeps
 * decoding while a scheduler looks at finished slots.  No counterpart in the
 * reference, whose BatchDecoder.finished synchronises the device
 * (engine.py:248-252) after every transcribe_many poll (transcribe.py:360-361). */
int32_t s2r_poll_finished_async(s2r_ctx* ctx, void* stream);

/* The flags of the last s2r_poll_finished_async: `*ready` = 1 and
 * `finished` [batch] filled once its copy has landed, else `*ready` = 0 (with
 * `wait` = 0 it never blocks; with `wait` != 0 it waits for that copy only,
 * not for the steps queued after it).  Fails with S2R_ESTATE without a
 * pending poll, and with S2R_EDEVICE if a kernel had reported an error. */
int32_t s2r_poll_finished_ready(s2r_ctx* ctx, uint8_t* finished, int32_t wait, int32_t* ready);

/* Asynchronous take: enqueue on `stream` the copy of slot's tokens, position
 * and end reason to host memory the engine owns, and free the slot at once
 * (its K/V pages return to the pool; a load of the slot queued after the copy
 * on the same stream is ordered behind it).  The tokens are read with
 * s2r_take_ready.  Replaces BatchDecoder.take (engine.py:254-262) for
 * schedulers that do not wait for the device. */
int32_t s2r_take_async(s2r_ctx* ctx, int32_t slot, void* stream);

/* The result of slot's s2r_take_async: as s2r_take (tokens ending in EOS,
 * end reason), with `*ready` = 0 while the copy has not landed (`wait` as in
 * s2r_poll_finished_ready).  S2R_ESTATE if the slot has no unread take. */
int32_t s2r_take_ready(s2r_ctx* ctx, int32_t slot, int64_t* tokens, int32_t capacity, int32_t* length,
                       int32_t* ended, int32_t wait, int32_t* ready);

/* Device address, element count and dtype code (0 f32, 1 bf16, 2 i64, 3 u8,
 * 4 f64, 5 i32) of a named engine buffer, for zero-copy views: "token",
 * "position", "finished", "ended", "in_shift", "shift_run", "payload",
 * "last_field", "incomplete", "g", "count", "target", "stop", "out",
 * "frames", "cross_k" / "cross_v" (layer 0's cross K/V, bf16
 * [batch][heads][frames][64], for inspection). Replaces reads of BatchDecoder.state / .out
 * (engine.py:138-144). */
int32_t s2r_get_buffer(s2r_ctx* ctx, const char* name, void** ptr, int64_t* numel, int32_t* dtype);

/* Run one decode step (it advances the slots like s2r_step) as a CUDA graph
 * with an event node after every kernel and no overlap between kernels, and
 * report per kernel
 * class — 0 qkv, 1 self attention, 2 self out-projection, 3 cross q,
 * 4 cross attention, 5 cross out-projection, 6 fc1, 7 fc2, 8 logits — the
 * summed device time in ms, the algorithmic bytes of one launch and the
 * launch count (host arrays of 9).  Synchronises `stream`.  Measurement only;
 * no counterpart in the reference. */
int32_t s2r_profile_step(s2r_ctx* ctx, float* ms, double* bytes, int32_t* launches, void* stream);

/* Kernel launches one decode step issues (for launch accounting). */
int32_t s2r_step_launches(s2r_ctx* ctx);

/* K/V pages of the pool that no slot holds. */
int32_t s2r_free_pages(s2r_ctx* ctx);

/* Grammar-masked greedy argmax over caller-provided device arrays, with no
 * device allocation: out[r] = argmax over v of (allowed[r][v] ?
 * logits[r][v] + bias[v] : -inf), lowest index on ties, 0 for a row with
 * nothing allowed.  `logits` [rows, vocab] float32, `bias` [vocab] float32 or
 * NULL, `allowed` [rows, vocab] uint8, `out` [rows] int64, all device memory.
 * For callers that cannot call cudaMalloc while decoding: a host whose pool
 * allocator reserves all device memory up front and forbids allocations
 * outside it, or a serving loop that must not stall the device (cudaFree
 * synchronises it, cudaMalloc may too).  Its cross-CTA scratch is
 * a static device array of 1024 rows + 1 counter, one copy per GPU that loads
 * the library; rows > 1024 fail with S2R_EINVAL.  Every call shares that
 * array, so calls that overlap on the GPU race; each call clears it first.
 * The first call on a device looks up the array's address and should come
 * before any stream capture on that device; the address is kept for the
 * process's life, so the entry point must not be called on a device after a
 * cudaDeviceReset of it.  A best allowed value of -inf also gives index 0,
 * and -0.0 ties with +0.0, as in torch.argmax.  Asynchronous on `stream`.
 * No counterpart in the reference (it computes this step with torch ops,
 * engine.py:316-317,349-350, inside its engine). */
int32_t s2r_masked_argmax_noalloc(const float* logits, const float* bias, const uint8_t* allowed, int32_t rows,
                                  int32_t vocab, int64_t* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* S2R_H */
