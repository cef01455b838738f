/*
 * llama_engine.h — C ABI of the B200 (sm_100a) engine for the llama3-signed-4bit token loop.
 *
 * Part 1 is the reference's ABI, unchanged in names, argument meaning and error behaviour, so
 * that the reference's callers (src/main.py ctypes bindings at :57-140, src/main.cpp,
 * tests/lm_eval_adapter.py) can load this library in place of the reference build.  Each entry
 * point cites the declaration it replaces (src/llama_engine.h) and the reference implementation
 * (src/llama_engine.cpp).
 *
 * Part 2 holds additive extensions (device selection, batched decode over independent
 * sequences, a device-resident greedy loop, the isolated block-128 GEMV).  No reference caller
 * needs them.
 *
 * Device residency: weights, KV caches, activations and logits live in GPU memory.
 * llama_engine_get_logits() returns a host pointer to a pinned mirror that is refreshed on
 * each call when the device logits are newer; the pointer stays valid until llama_engine_free(),
 * and its contents are current as of the last get_logits() call.
 *
 * Threading: one engine handle must not be used from two host threads at once (the reference
 * shares scratch buffers per handle in the same way).  Separate handles are independent.
 */
#ifndef LLAMA_ENGINE_H
#define LLAMA_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* llama_engine_t;     /* src/llama_engine.h:12 */
typedef void* llama_tokenizer_t;  /* src/llama_engine.h:13 */

/* ---------------------------------------------------------------------------------------- */
/* Part 1: the reference ABI                                                                 */
/* ---------------------------------------------------------------------------------------- */

/* src/llama_engine.h:20, impl src/llama_engine.cpp:1051-1059.  Loads an LLM4S128 file onto
 * CUDA device 0 (or $LLAMA_ENGINE_DEVICE).  Returns NULL on any failure: missing file, bad
 * magic, a file shorter than its header implies, unsupported geometry, or a CUDA error. */
llama_engine_t llama_engine_create(const char* model_path);

/* src/llama_engine.h:23, impl :1061-1065.  NULL is a no-op. */
void llama_engine_free(llama_engine_t engine);

/* src/llama_engine.h:26, impl :1067-1071 and :930-933.  A no-op: KV positions are simply
 * overwritten from pos 0 by the next sequence, as in the reference. */
void llama_engine_reset(llama_engine_t engine);

/* src/llama_engine.h:29-36, impl :1073-1110.  0 for a NULL handle; get_max_seq_len ignores
 * the handle and returns 8192 (MAX_SEQ_LEN, src/llama_engine.cpp:26). */
int32_t llama_engine_get_num_layers(llama_engine_t engine);
int32_t llama_engine_get_dim(llama_engine_t engine);
int32_t llama_engine_get_ffn_dim(llama_engine_t engine);
int32_t llama_engine_get_vocab_size(llama_engine_t engine);
int32_t llama_engine_get_num_heads(llama_engine_t engine);
int32_t llama_engine_get_num_kv_heads(llama_engine_t engine);
int32_t llama_engine_get_head_dim(llama_engine_t engine);
int32_t llama_engine_get_max_seq_len(llama_engine_t engine);

/* src/llama_engine.h:40, impl :1112-1116 and :935-1042.  Runs one token through all layers
 * at position pos of sequence slot 0, writing its K/V rows, and the lm_head when
 * compute_logits != 0.  pos >= 8192 is a silent no-op; an out-of-range token id is replaced by
 * 0 (both as in the reference).  Returns 0, or -1 for a NULL handle or a CUDA error.  The call
 * is stream-ordered: it returns once the work is queued on the GPU. */
int llama_engine_forward_token(llama_engine_t engine, int32_t token_id, size_t pos, int compute_logits);

/* src/llama_engine.h:44, impl :1118-1127.  Same result as count forward_token calls at
 * start_pos..start_pos+count-1 with logits only for the last one (if compute_last_logits).
 * Returns -1 for a NULL handle or NULL token_ids. */
int llama_engine_prefill(llama_engine_t engine, const int32_t* token_ids, size_t count, size_t start_pos, int compute_last_logits);

/* src/llama_engine.h:47, impl :1129-1133 and :784-839.  temperature <= 0.01: greedy argmax
 * (first index among equal maxima).  Otherwise the logits are overwritten in place with
 * probabilities (temperature, softmax) on the device, 64 candidates are chosen by the
 * reference's insertion walk (ids 0..63 first, then every id that beats the list's last entry,
 * replayed on the device), and libc rand() draws within the top_p mass on the host, as in the
 * reference.  0 for a NULL handle. */
int32_t llama_engine_sample(llama_engine_t engine, float temperature, float top_p);

/* src/llama_engine.h:50, impl :1135-1138.  Host pointer to vocab_size floats (see top). */
const float* llama_engine_get_logits(llama_engine_t engine);

/* src/llama_engine.h:53, impl :1140-1144 and :182-220.  Dequantises embedding row token_id
 * (of the tied lm_head) into out_x[dim] on the host side.  No-op for NULL arguments or an
 * out-of-range token id. */
void llama_engine_dequantize_embedding(llama_engine_t engine, size_t token_id, float* out_x);

/* src/llama_engine.h:59-62, impl :1146-1178.  Byte-level BPE tokenizer over a HF
 * tokenizer.json (host code; not on the GPU path).  encode returns the number of ids written
 * (0 on bad arguments); decode returns a string owned by the tokenizer, valid until the next
 * decode call on it ("" for unknown ids). */
llama_tokenizer_t llama_tokenizer_create(const char* tokenizer_path);
void llama_tokenizer_free(llama_tokenizer_t tokenizer);
int llama_tokenizer_encode(llama_tokenizer_t tokenizer, const char* text, int32_t* out_tokens, int max_tokens);
const char* llama_tokenizer_decode(llama_tokenizer_t tokenizer, int32_t token_id);

/* ---------------------------------------------------------------------------------------- */
/* Part 2: extensions (no counterpart in the reference ABI)                                  */
/* ---------------------------------------------------------------------------------------- */

/* Like llama_engine_create, on CUDA device `device`, with KV caches for `max_batch`
 * independent sequence slots of `max_seq_len` positions each (max_seq_len <= 8192; 0 means
 * 8192).  Slot 0 is the sequence used by the Part-1 calls.  NULL on failure. */
llama_engine_t llama_engine_create_ex(const char* model_path, int device, int max_batch, int max_seq_len);

/* Message of the last failure on this handle (or of the last failed create when engine is
 * NULL).  Never NULL. */
const char* llama_engine_last_error(llama_engine_t engine);

/* Device-resident greedy loop, equal to n_steps x { forward_token(tok, pos, 1); tok =
 * sample(0, .) ; pos++ } starting from (first_token, start_pos) on slot 0.  Writes the n_steps
 * sampled ids to out_tokens (host memory).  Returns 0, or -1 on error / pos overflow. */
int llama_engine_generate_greedy(llama_engine_t engine, int32_t first_token, size_t start_pos,
                                 int32_t n_steps, int32_t* out_tokens);

/* Batched decode: one step for n independent sequences.  Row i feeds tokens[i] at positions[i]
 * into sequence slot slots[i] (slots < max_batch; positions < max_seq_len).  Host arrays.
 * Rows of one slot must come in increasing position order; each row attends to its slot's
 * cache up to its own position, including rows of the same call.  n <= max_batch, or, on the
 * tensor-core batched path (llama_engine_batch_path() == 1) and without logits, up to
 * max(max_batch, prefill chunk) rows, e.g. several prompt positions of many slots at once.
 * compute_logits != 0 also runs the lm_head for every row.  Stream-ordered: returns once the
 * step is queued (0), or -1 on bad arguments; a device error of the step is reported by the next
 * call that waits for it (argmax_batch, get_logits_batch). */
int llama_engine_forward_batch(llama_engine_t engine, const int32_t* tokens, const int32_t* positions,
                               const int32_t* slots, int n, int compute_logits);

/* Greedy ids (first index among equal maxima) of the n rows of the last forward_batch.
 * Waits for the step; -1 on bad arguments or a device error. */
int llama_engine_argmax_batch(llama_engine_t engine, int32_t* out_tokens, int n);

/* Host pointer to the logits of row `row` of the last forward_batch (vocab_size floats,
 * refreshed by this call).  NULL on error. */
const float* llama_engine_get_logits_batch(llama_engine_t engine, int row);

/* Isolated block-128 GEMV, y[m][n] = sum_k w[n][k] * x[m][k] with w = min + q*step, for the M
 * rows of x (1 <= M <= 8), all pointers in device memory with the LLM4S128 matrix layout
 * (nibbles[N*K/2], step_bf16[N*K/128], min_bf16[N*K/128]).  K % 128 == 0.  `stream` is a
 * cudaStream_t (NULL = legacy default stream).  Counterpart of the reference's file-local
 * signed_4bit_b128_gemv (src/llama_engine.cpp:233-357), which receives the block sums of x
 * precomputed; here they are computed inside the kernel.  `nibbles` and `x` must be 16-byte
 * aligned.  Returns 0, or -1 on bad arguments / launch error. */
int llama_b128_gemv(const uint8_t* nibbles, const uint16_t* step_bf16, const uint16_t* min_bf16,
                    int N, int K, const float* x, int M, float* y, void* stream);

/* Same product for 1 <= M <= 4096 rows on the tensor-core (tcgen05) kernel that the batched
 * decode and prefill use: the weights become exact bf16 codes, x is split into bf16 hi + lo
 * parts, fp32 accumulation per 128-block, scales applied in fp32.  K in {2048, 4096, 6144,
 * 8192}.  Builds its working layout in temporary device buffers and returns after the result
 * is complete (synchronises `stream`), so it is meant for tests and measurements.  Needs an
 * sm_100 device.  Returns 0, or -1 on bad arguments / device error. */
int llama_b128_gemm(const uint8_t* nibbles, const uint16_t* step_bf16, const uint16_t* min_bf16,
                    int N, int K, const float* x, int M, float* y, void* stream);

/* Host-side planner of the tensor-core GEMM's work units (no device work; extension with no
 * counterpart in the reference, which has no tensor-core path): for a GEMM of `tiles` 128-row
 * weight tiles, `kb` 128-wide K blocks and `img_tiles` 64-token activation tiles on `num_sms` SMs,
 * writes out[0] = unit form (1: 64-token units, 2: 128-token units over two tiles), out[1] =
 * token groups (units along the tokens), out[2] = K splits, out[3] = K blocks per split.
 * splits_req > 0 fixes the splits (the gate-up and lm_head GEMMs use 1).  The batched steps and
 * llama_b128_gemm launch what this returns.  Returns 0, or -1 for arguments out of range. */
int llama_b128_gemm_plan(int num_sms, int tiles, int kb, int img_tiles, int splits_req, int32_t* out);

/* Log-likelihood of a token run, for scoring consumers such as the reference's lm-eval adapter
 * (tests/lm_eval_adapter.py:111-229, which calls forward_token + get_logits per token and forms
 * log_softmax on the host).  Runs tokens[0..n) through slot 0 at positions start_pos.. (in
 * chunks of up to 256 on the tensor-core batched path, else token by token), and for
 * i in [0, n-1) writes out_logprobs[i] = log P(tokens[i+1] | tokens[..i]) computed on the device as
 * (l[t] - max l) - log(sum exp(l - max l)) over the fp32 logits, and, when out_greedy is not
 * NULL, out_greedy[i] = 1 if tokens[i+1] is the greedy id of those logits (first index among
 * equal maxima), else 0.  Afterwards the current logits are those of tokens[n-1], as after
 * prefill(..., compute_last_logits = 1).  Out-of-range ids count as id 0, as in forward_token.
 * Returns 0, or -1 on bad arguments (NULL pointers, n < 2, start_pos + n > max_seq_len) or a
 * device error. */
int llama_engine_score_tokens(llama_engine_t engine, const int32_t* tokens, size_t n, size_t start_pos,
                              float* out_logprobs, int32_t* out_greedy);

/* Which implementation runs the slot-0 token steps: 1 = the persistent token-step kernel (one
 * cooperative launch per forward_token, or per whole generate_greedy call; used for dim 2048
 * and ffn_dim in {2048, 4096, 8192}), 0 = the per-phase kernel chain in a CUDA graph (any other
 * supported geometry, or LLAMA_B200_PERSISTENT=0 at create time), 2 = the 2-way tensor-parallel
 * engine (llama_engine_create_tp).  -1 for a NULL handle. */
int llama_engine_decode_path(llama_engine_t engine);

/* Which implementation runs prefill (2 or more tokens) and llama_engine_forward_batch: 1 = the
 * token-batched path with tensor-core (tcgen05) GEMMs (sm_100 devices, dim and ffn_dim
 * multiples of 2048, 4 q heads per kv head; LLAMA_B200_BATCHED=0 at create time turns it off),
 * 0 = token by token through the decode path.  -1 for a NULL handle. */
int llama_engine_batch_path(llama_engine_t engine);

/* Diagnostics for the persistent kernel: enable = 1 starts recording a phase trace of the first
 * token of each following launch (globaltimer timestamps per CTA at every phase's start, after
 * its dependency wait, after staging and at its end), 0 stops, 2 copies up to max_entries
 * (time_ns, tag) pairs laid out as [cta][1024] into `out` and returns the count.  Tags:
 * (event << 16) | (phase << 8) | layer, event 1..4; 0xFFFF0000 marks a token start.
 * Returns -1 when the engine does not use the persistent kernel. */
int llama_engine_trace(llama_engine_t engine, int enable, unsigned long long* out, int max_entries);

/* The cudaStream_t on which the engine enqueues all of its work (for CUDA-event timing and
 * stream ordering by the caller).  NULL for a NULL handle. */
void* llama_engine_get_stream(llama_engine_t engine);

/* Diagnostics: enqueues `iters` launches of one phase of the token step on the engine stream,
 * cycling through the layers (so consecutive launches read different weights), between two
 * CUDA events, and returns the average time per launch in *avg_ms.  Phases: "qkv", "attn",
 * "oproj", "gateup", "down", "lmhead", "step" (one whole token, graph launch).  Returns 0 or -1.
 * Activations are whatever the last step left; the numbers are timings only. */
int llama_engine_profile_phase(llama_engine_t engine, const char* phase, int iters, float* avg_ms);

/* 2-way tensor-parallel batch-1 variant (no counterpart in the reference, which runs on one
 * CPU): one process per GPU, each creating its engine with the same NCCL unique id.  Rank 0
 * makes the id with llama_engine_tp_unique_id (writes 128 bytes; returns 0, or -1 when NCCL
 * cannot be loaded) and the caller passes it to the other rank.  Each rank holds half of every
 * layer (q heads and kv heads by halves, W_o and W_down by column halves, W_gate / W_up and the
 * lm_head by row halves); per layer the o-proj and down partial sums are all-reduced (NCCL over
 * NVLink) and the greedy id is the better of the two ranks' candidates.  Both ranks must make
 * the same calls in the same order: forward_token, prefill (token by token), sample with
 * temperature <= 0.01, get_logits (all 128,256 logits, gathered on both ranks),
 * generate_greedy.  Batched calls are not available on this engine.  NULL on failure. */
int llama_engine_tp_unique_id(void* out_id, int len);
llama_engine_t llama_engine_create_tp(const char* model_path, int device, int rank, int world, const void* unique_id,
                                      int max_seq_len);

/* Opt-in llama3 RoPE frequency scaling.  By default the engine uses the reference's table,
 * theta_i = 500000^(-2i/64) without scaling (src/llama_engine.cpp:908-917), which is what parity
 * with the reference requires.  With factor > 0 the table is rebuilt with the "llama3" rescaling
 * of the reference's models/config.json:26-32 (factor 32, low_freq_factor 1, high_freq_factor 4,
 * original_max_position 8192 there), which its Hugging Face path applies (chat.py:42): wavelengths
 * longer than original/low_freq_factor are stretched by factor, shorter than
 * original/high_freq_factor are kept, and the band between is blended.  factor <= 0 restores the
 * reference's table.  Waits for the engine's queued work first.  Returns 0, or -1 on bad
 * parameters or a device error. */
int llama_engine_set_rope_scaling(llama_engine_t engine, float factor, float low_freq_factor,
                                  float high_freq_factor, int original_max_position);

/* The RoPE table the engine would use for those parameters (host only): cos_out and sin_out
 * receive [n_pos][32] floats, n_pos <= 8192.  Returns 0, or -1 on bad arguments. */
int llama_engine_rope_table(float factor, float low_freq_factor, float high_freq_factor, int original_max_position,
                            int n_pos, float* cos_out, float* sin_out);

/* Diagnostics, host only (no device is touched): builds the persistent kernel's work schedule
 * for a model geometry and a grid of `grid` CTAs, and checks it the way the kernel reads it
 * (every 16-row tile of every phase handled by exactly one CTA with that tile's records of the
 * right matrices, records consumed in stream order, segments in phase order, every attention
 * head once per layer, shared-memory capacity limits).  Returns 0 when the schedule is valid,
 * -1 otherwise with a message in err (err_len bytes, may be NULL). */
int llama_engine_check_schedule(int layers, int dim, int ffn_dim, int vocab_size, int num_heads, int num_kv_heads,
                                int grid, char* err, int err_len);

/* Test hook for the bounded device waits: sets the time bound of every wait of the persistent
 * kernel, the tensor-core GEMM and the prefill attention to wait_ns (0 restores the default of
 * 2 s), and with expire_code != 0 makes the next launches wait on a device word that nothing
 * writes, so that the wait runs out: the persistent kernel's CTA 0 at the start of a launch, the
 * GEMM's MMA issuer before its first block; expire_code = 20 instead expires only the prefill
 * attention kernel (its MMA-issuing thread, after the first K / V tile copies are in flight),
 * and the GEMMs then keep the default bound, so that only the attention's wait runs out.  The launch
 * then drains and the next waiting call fails with the timeout reported; expire_code = 0 turns
 * that off again and clears the recorded error so the engine can be used again.  Returns 0, or
 * -1 for a NULL handle. */
int llama_engine_debug_waits(llama_engine_t engine, unsigned long long wait_ns, int expire_code);

/* Greedy argmax of n device-resident fp32 logits that allocates no memory: writes the first
 * index among the maxima (values <= -1e30 and NaN never win; 0 when none qualifies, the
 * reference's rule at src/llama_engine.cpp:785-792) to *out_index (device memory).  No
 * counterpart in the reference ABI.  It is for callers that cannot allocate device memory while
 * running (a fixed memory budget reserved at start-up, or a decode loop that cannot afford the
 * device synchronisation a cudaMalloc may cause): its scratch is a fixed 8 KB device array inside
 * this library, held by every GPU that loads the library until the process exits.  The first
 * call on a device looks up that array's device address; make that first call before any stream
 * capture.  All calls share the array, so calls that overlap on the GPU (different streams
 * without ordering) race; calls on one stream are safe.  n <= 16,777,216.  Returns 0, -1 on bad
 * arguments or a launch error, -2 when n exceeds the maximum. */
int llama_b128_argmax_noalloc(const float* logits, int n, int32_t* out_index, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LLAMA_ENGINE_H */
