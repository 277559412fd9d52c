/* strands-decider B200: the C ABI of the sequence-mixing forward.
 *
 * The drop-in boundary for the reference's torso engine (strands-decider-rs, `src/engine.rs`): a
 * Rust host binds these with `extern "C"` declarations in place of `Engine::load` /
 * `Engine::forward` / `Snapshot`, and the rest of `Decider` (tokenizer, prompt, head, `ask_all`)
 * stays as it is. Plain pointers and sizes only; host buffers unless a name says
 * `dev`. Every call returns SD_OK or a negative code; the message of the last failure is in
 * sd_engine_last_error(engine) (or sd_last_error() for calls without an engine), as the
 * reference's `Error(String)` (`src/lib.rs:23-44`) carries it. An engine is used by one host thread
 * at a time (the reference's `&mut self`, `src/engine.rs:529`); engines on different GPUs run
 * concurrently.
 */
#ifndef SD_B200_H
#define SD_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SD_OK 0
#define SD_ERR_INVALID (-1) /* bad argument: context, row range, token id (`src/engine.rs:530-537`) */
#define SD_ERR_IO (-2)      /* a model file is missing or short */
#define SD_ERR_FORMAT (-3)  /* manifest/tensor format not supported (`src/engine.rs:245-250`) */
#define SD_ERR_CUDA (-4)    /* a CUDA call failed (including out of memory) */
#define SD_ERR_KERNEL (-5)  /* a kernel reported an error (a bounded wait ran out, a bad shape) */

#define SD_CONTEXT 4096 /* tokens of KV cache and RoPE table (`src/engine.rs:16`) */

typedef struct sd_engine sd_engine;
typedef struct sd_snapshot sd_snapshot;
typedef struct sd_head sd_head;
typedef struct sd_qweight sd_qweight;

/* Replaces `Engine::load(dir, &Manifest)` (`src/engine.rs:175-303`): reads `manifest.json`, the
 * weight shards and the embedding rows of a model directory onto GPU `device`. */
int sd_engine_create(const char* model_dir, int device, sd_engine** out);
void sd_engine_destroy(sd_engine* e);
/* Sizes the engine's working memory (activations, staging, pinned buffers) for passes of up to
 * max_tokens tokens, max_seqs sequences and max_rows hidden rows, so that no later call within those
 * bounds allocates (an allocation waits for the engine's queued work). A server calls it once at
 * start-up; without it the buffers grow on demand. */
int sd_engine_reserve(sd_engine* e, int32_t max_tokens, int32_t max_seqs, int32_t max_rows);
/* `Engine::hidden_size` (`src/engine.rs:305-307`). */
int sd_engine_hidden_size(const sd_engine* e);
const char* sd_engine_last_error(const sd_engine* e);
const char* sd_last_error(void);

/* Replaces `Engine::forward(ids, rows, cache, keep, timed)` (`src/engine.rs:529-662`): runs the torso
 * over `n_ids` new tokens after the prefix in `cache` (NULL: none), writes the final hidden rows
 * `rows` (indices into ids) to `hidden_out` [n_rows][hidden_size] f32 and, when `keep`, a snapshot
 * covering the prefix and these tokens to `*snapshot_out`. `gpu_ms_out` (may be NULL) receives the
 * device time of the forward, as the reference's timestamp queries measure it. */
int sd_forward(sd_engine* e, const uint32_t* ids, int32_t n_ids, const int32_t* rows, int32_t n_rows,
               const sd_snapshot* cache, int32_t keep, float* hidden_out, sd_snapshot** snapshot_out,
               double* gpu_ms_out);

/* The batched fork: `nq` questions, each a forward of lens[b] new tokens continuing the snapshot
 * `cache`, in one pass (it replaces the serial loop of `Decider::ask_all`, `src/lib.rs:192-198`,
 * whose every question is an `Engine::forward(ids, rows, Some(&snapshot), false, ..)`). ids: the
 * questions' tokens back to back (sum of lens); rows: each question's rows (indices into its own
 * tokens, nrows[b] of them), back to back; hidden_out: [sum of nrows][hidden_size] f32 in the same
 * order. The results equal nq separate sd_forward calls up to f32 summation order. The snapshot is
 * read in place and not changed. gpu_ms_out (may be NULL): device time of the pass. */
int sd_forward_fork(sd_engine* e, const sd_snapshot* cache, const uint32_t* ids, const int32_t* lens, int32_t nq,
                    const int32_t* rows, const int32_t* nrows, float* hidden_out, double* gpu_ms_out);
/* sd_forward_fork with the token ids already on the GPU (ids_dev) and the hidden rows written to
 * hidden_dev [sum of nrows][hidden_size] f32, asynchronous on the engine's stream (lens, rows and
 * nrows stay host arrays: they shape the pass). Token ids are checked on the device; errors surface
 * at the next sd_engine_synchronize. */
int sd_forward_fork_dev(sd_engine* e, const sd_snapshot* cache, const uint32_t* ids_dev, const int32_t* lens, int32_t nq,
                        const int32_t* rows, const int32_t* nrows, float* hidden_dev);
/* The batched fork across requests: question b continues caches[b] (any snapshots of this engine,
 * of any lengths; several questions may share one), so the questions of many `Decider::ask_all`
 * calls run as one pass, which is how a server answers concurrent requests. Otherwise as
 * sd_forward_fork / sd_forward_fork_dev (at most 4096 questions and 65536 tokens per call). */
int sd_forward_fork_multi(sd_engine* e, const sd_snapshot* const* caches, const uint32_t* ids, const int32_t* lens,
                          int32_t nq, const int32_t* rows, const int32_t* nrows, float* hidden_out, double* gpu_ms_out);
int sd_forward_fork_multi_dev(sd_engine* e, const sd_snapshot* const* caches, const uint32_t* ids_dev, const int32_t* lens,
                              int32_t nq, const int32_t* rows, const int32_t* nrows, float* hidden_dev);
/* Many `Engine::forward` calls in one pass: sequence b is lens[b] new tokens continuing caches[b]
 * (NULL entry, or a NULL caches array: a fresh sequence, as `Engine::forward(.., None, ..)`), its
 * rows (nrows[b] of them, indices into its own tokens) written to hidden_out in order; with `keep`,
 * snapshots_out[b] receives a snapshot covering caches[b]'s tokens and these (free each with
 * sd_snapshot_free). The results equal nseq separate sd_forward calls up to f32 summation order;
 * the source snapshots are read and not changed. This is how a server prefills the states of
 * concurrent requests: the GEMMs see every sequence's rows at once, and the gated-delta scans and
 * attention of all sequences run side by side. At most 4096 sequences and 65536 tokens per call. */
int sd_forward_batch(sd_engine* e, const sd_snapshot* const* caches, const uint32_t* ids, const int32_t* lens, int32_t nseq,
                     const int32_t* rows, const int32_t* nrows, int32_t keep, float* hidden_out, sd_snapshot** snapshots_out,
                     double* gpu_ms_out);
/* sd_forward_batch with the ids on the GPU and the rows to hidden_dev, asynchronous on the engine's
 * stream (the new snapshots are returned at once and usable by later calls on the engine). */
int sd_forward_batch_dev(sd_engine* e, const sd_snapshot* const* caches, const uint32_t* ids_dev, const int32_t* lens,
                         int32_t nseq, const int32_t* rows, const int32_t* nrows, int32_t keep, float* hidden_dev,
                         sd_snapshot** snapshots_out);

/* `Snapshot::len` (`src/engine.rs:80-87`): tokens covered. A snapshot is immutable and can seed
 * any number of forwards on the engine that made it; free it with sd_snapshot_free. */
int32_t sd_snapshot_len(const sd_snapshot* s);
void sd_snapshot_free(sd_snapshot* s);

/* `Engine::forward` on device memory, asynchronous on the engine's stream (sd_engine_stream): ids_dev
 * [n_ids] u32 and rows_dev [n_rows] i32 already on the GPU, hidden rows to hidden_dev
 * [n_rows][hidden_size] f32. Token ids and rows are checked on the device; errors surface at the
 * next sd_engine_synchronize. A snapshot made here can be used by later calls at once (the work is
 * stream-ordered). The caller keeps ids_dev/rows_dev alive until the work completes. */
int sd_forward_dev(sd_engine* e, const uint32_t* ids_dev, int32_t n_ids, const int32_t* rows_dev, int32_t n_rows,
                   const sd_snapshot* cache, int32_t keep, float* hidden_dev, sd_snapshot** snapshot_out);
/* Waits for the engine's queued work; returns the first error a kernel reported since the last call. */
int sd_engine_synchronize(sd_engine* e);
/* A self-test of the failure path that no valid input reaches (this call has no counterpart in the
 * reference, which returns device errors as `Err`, src/engine.rs:648-651): on the engine's stream, one
 * warp of a small kernel waits on a barrier phase that nothing completes and gives up after limit_us
 * microseconds (1..1000000), recording a timeout in the engine's error word and setting its CTA's abort
 * flag, while a second warp waiting with the kernels' full 2 s limit leaves on that flag, as every
 * warp-specialised kernel of the library does. Nothing faults; the call returns SD_ERR_KERNEL with the
 * timeout's message, as a forward whose kernel gave up would, and the engine stays usable. */
int sd_engine_selftest_wait(sd_engine* e, int32_t limit_us);
/* The engine's CUDA stream (a cudaStream_t), for callers that order their own work after it. */
void* sd_engine_stream(const sd_engine* e);
/* Kernels of this library the engine has launched since it was created. */
int64_t sd_engine_launches(const sd_engine* e);

/* Diagnostics: when `host_buf` is set, each following forward writes the residual stream after each
 * layer (x + y, [n_layers][n_ids][hidden_size] f32) there; `floats` is its capacity. NULL stops. */
int sd_engine_set_trace(sd_engine* e, float* host_buf, size_t floats);
int sd_engine_num_layers(const sd_engine* e);

/* Per-kernel device time, as the reference's `Engine::profile` (`src/engine.rs:665-711`) gives it per
 * dispatch label: while enabled, every launch is bracketed by CUDA events on the engine's stream.
 * sd_engine_profile_get returns, per kind, the summed milliseconds, the launches and the summed
 * algorithmic work (FLOPs for SD_PROF_GEMM and SD_PROF_ATTN, bytes for the others) since the last
 * enable. Reading synchronizes. */
#define SD_PROF_GEMM 0  /* dequantizing matmuls (work: 2 m n k FLOPs) */
#define SD_PROF_ATTN 1  /* attention (work: 4 hd hq causal pairs FLOPs) */
#define SD_PROF_GDN 2   /* gated delta rule (work: q,k,v,gates,o,state bytes) */
#define SD_PROF_OTHER 3 /* norms, conv, gates, q/k prep, embedding (work: bytes moved) */
#define SD_PROF_KINDS 4
int sd_engine_profile(sd_engine* e, int32_t enable);
int sd_engine_profile_get(sd_engine* e, int32_t kind, double* ms, int64_t* launches, double* work);

/* Replaces `Head::load` and `Head::probs` (`src/head.rs:25-77`): the pointer head in f64 on the
 * host. `hidden` is [n_rows][d] = [option 0 .. option n-2, answer]; writes n_rows - 1 probabilities. */
int sd_head_load(const char* safetensors_path, sd_head** out);
void sd_head_free(sd_head* h);
int sd_head_probs(const sd_head* h, const float* hidden, int32_t n_rows, int32_t d, double temperature, double* probs_out);
/* `Head::probs` on the GPU, for many questions at once, asynchronous on the engine's stream (f64 as
 * on the host; sums in tree order, so equal to sd_head_probs to f64 rounding). hidden_dev holds the
 * questions' rows back to back as the engine's _dev calls write them (question i: n_rows[i] rows,
 * options then answer, hidden_size f32 each; a rotated torso's rows are mapped back on the device);
 * temperatures[i] (host) is question i's; probs_dev gets sum(n_rows[i] - 1) f64, question after
 * question (at most 65535 questions per call). The head's weights go to the engine's device on first
 * use; sd_head_free releases them (after the device's queued work). */
int sd_head_probs_dev(sd_engine* e, const sd_head* h, const float* hidden_dev, const int32_t* n_rows, int32_t n_questions,
                      const double* temperatures, double* probs_dev);
/* sd_forward_fork_multi with the pointer head on the GPU: the questions' hidden rows never leave the
 * device, only their probabilities come back (probs_out, host, sum(n_rows[i] - 1) f64; every
 * question needs 2 or more rows: its options and its answer). Synchronous. The question loop of
 * `Decider::run` (`src/lib.rs:191-198`: a forward from the prefix snapshot, then `Head::probs`, per
 * question) as one call. */
int sd_forward_fork_multi_probs(sd_engine* e, const sd_snapshot* const* caches, const uint32_t* ids, const int32_t* lens,
                                int32_t n_questions, const int32_t* rows, const int32_t* n_rows, const sd_head* h,
                                const double* temperatures, double* probs_out);

/* A request's state and its questions in one packed pass (instead of a forward, then a fork): sequence
 * b continues caches[b] (caches may be null; null entries: a fresh sequence) or, with parent[b] >= 0,
 * the earlier sequence parent[b] of the same call, which must itself have no parent (parent[b] = -1
 * otherwise; a sequence with a parent has no snapshot of its own). Each layer writes the parents'
 * recurrent states, conv histories and keys/values before their children read them, so the children
 * see what a kept snapshot of the parent would hold (`Engine::forward` with a cache,
 * src/engine.rs:529-662, and the question loop of `Decider::ask_all`, src/lib.rs:192-198). No
 * snapshots come out. rows / nrows: output rows per sequence (indices into its own tokens; a
 * parent's may be none); hidden_out [sum nrows][d] f32. */
int sd_forward_tree(sd_engine* e, const sd_snapshot* const* caches, const int32_t* parent, const uint32_t* ids,
                    const int32_t* lens, int32_t nseq, const int32_t* rows, const int32_t* nrows, float* hidden_out);

/* sd_forward_tree with the ids on the GPU and the rows written to hidden_dev, queued on the engine's
 * stream (as sd_forward_batch_dev). */
int sd_forward_tree_dev(sd_engine* e, const sd_snapshot* const* caches, const int32_t* parent, const uint32_t* ids_dev,
                        const int32_t* lens, int32_t nseq, const int32_t* rows, const int32_t* nrows, float* hidden_dev);

/* sd_forward_tree, then the pointer head on the GPU over the sequences that have rows (nrows[b] = 0,
 * or 2 or more: the options, then the answer row), as sd_forward_fork_multi_probs; probs_out gets
 * their probabilities in sequence order (nrows[b] - 1 each). temperatures: one per sequence (those
 * of sequences without rows are not read). */
int sd_forward_tree_probs(sd_engine* e, const sd_snapshot* const* caches, const int32_t* parent, const uint32_t* ids,
                          const int32_t* lens, int32_t nseq, const int32_t* rows, const int32_t* nrows, const sd_head* h,
                          const double* temperatures, double* probs_out);

/* The Decider on the engine (the reference's `Decider`, `src/lib.rs:100-209`): tokenizer, prompt,
 * torso, pointer head and answers in the library (C++). */
typedef struct sd_decider sd_decider;
typedef struct sd_tokenizer sd_tokenizer;
/* `Decider::load` (`src/lib.rs:120-134`): tokenizer.json, the torso (sd_engine_create on `device`),
 * head.safetensors and hobson_config.json of a model directory. Failure: sd_host_last_error(). */
int sd_decider_load(const char* model_dir, int device, sd_decider** out);
void sd_decider_free(sd_decider* d);
/* `Decider::evaluate` / `ask_all` (`src/lib.rs:141-208`) on a System One request
 * (`Request::from_json`, `src/lib.rs:46-63`: {"state": content, "questions": {name: question}}):
 * writes the response body (`Response::to_json`, `src/lib.rs:78-87`: model, answers by name, usage) to
 * *response_json, a NUL-terminated string the caller frees with sd_string_free. Several questions
 * share one encoding of the state: a snapshot, then one batched fork per 32 questions. */
int sd_decider_ask_all(sd_decider* d, const char* request_json, char** response_json);
/* Many requests at once (a JSON array of requests as sd_decider_ask_all takes them), as a server
 * answers concurrent ones: the requests' states in packed passes (sd_forward_batch), then all their
 * questions in packed forks with the pointer head on the GPU (sd_forward_fork_multi_probs). Writes a
 * JSON array in the same order: each request's response body, equal to its own sd_decider_ask_all up
 * to f32 summation order, or {"error": message} for a request that failed. The call itself fails
 * only on a malformed array. */
int sd_decider_ask_batch(sd_decider* d, const char* requests_json, char** responses_json);
const char* sd_decider_last_error(const sd_decider* d);
const char* sd_host_last_error(void);
void sd_string_free(char* s);

/* `Tokenizer::from_json` / `encode` (`src/tokenizer.rs:84-155`) on their own: `text` (len bytes of
 * UTF-8) to ids and byte offsets ([n][2], into the NFC text); at most `cap` are written, *n_out is the
 * full count. */
int sd_tokenizer_load(const char* tokenizer_json_path, sd_tokenizer** out);
void sd_tokenizer_free(sd_tokenizer* t);
int sd_tokenizer_encode(const sd_tokenizer* t, const char* text, size_t len, uint32_t* ids, uint32_t* offsets, int64_t cap,
                        int64_t* n_out);
/* Many texts (texts[i], lens[i] bytes) encoded on up to `threads` host threads (0: one per hardware
 * thread, at most 16), as a server tokenizes concurrent requests; sd_decider_ask_batch prepares its
 * requests the same way. counts[i] gets text i's token count; ids and offsets are written text after
 * text, at most `cap` tokens in all. Equal to n sd_tokenizer_encode calls. A text that fails fails
 * the call (the first by index names it). */
int sd_tokenizer_encode_batch(const sd_tokenizer* t, const char* const* texts, const size_t* lens, int64_t n, int32_t threads,
                              uint32_t* ids, uint32_t* offsets, int64_t cap, int64_t* counts);
/* Prompt rendering (`src/prompt.rs:159-200`) of {"state": content, "questions": [question, ...]}:
 * writes {"state": text, "questions": [{"text": text, "spans": [[begin, end], ...]}]} (byte ranges of
 * the option lines) to *out_json (free with sd_string_free). */
int sd_prompt_render(const char* request_json, char** out_json);

/* Kernel-level entry points on device memory, on CUDA stream `stream` (a cudaStream_t; NULL: the
 * legacy default stream). They replace single dispatches of the reference's plan
 * (`src/engine.rs:396-524`) and serve the isolated benchmarks. */

/* `kernels::attn` (`src/kernels.rs:453-541`): causal GQA attention with the sigmoid output gate.
 * q_dev [hq][l][hd] f16; k_dev/v_dev [hk][lt][hd] f16 with this call's rows at p..p+l-1; gate at
 * gate_dev[t * gstride + goff + h * gstep + d] f16 (NULL: ungated); out_dev [l][hq * hd] f16. hd = 256. */
int sd_attention(const void* q_dev, const void* k_dev, const void* v_dev, const void* gate_dev, int32_t gstride,
                 int32_t goff, int32_t gstep, void* out_dev, int32_t l, int32_t p, int32_t lt, int32_t hq, int32_t hk,
                 int32_t hd, void* stream);

/* sd_attention over `batch` independent sequences in one launch (the reference dispatches `attn` once
 * per sequence): q_dev [batch][hq][l][hd], k_dev/v_dev [batch][hk][lt][hd], gate rows and out rows
 * batch-major ([batch][l][gstride], [batch][l][hq * hd]); everything else as sd_attention. */
int sd_attention_batch(const void* q_dev, const void* k_dev, const void* v_dev, const void* gate_dev, int32_t gstride,
                       int32_t goff, int32_t gstep, void* out_dev, int32_t batch, int32_t l, int32_t p, int32_t lt, int32_t hq,
                       int32_t hk, int32_t hd, void* stream);

/* sd_attention on the mma.sync kernel with the keys split across `splits` CTAs per (query block,
 * head) (0: the engine's choice, which splits only when the query blocks x heads leave SMs idle, as
 * for a short continuation over a long prefix); each split's partial result is merged by a second
 * kernel. ws_dev: f32 workspace of splits x hq x l x (hd + 2) floats (16-byte aligned; unused with one
 * split). sd_attention itself takes the tcgen05 kernel for l >= 128 (query blocks of 128). */
int sd_attention_split(const void* q_dev, const void* k_dev, const void* v_dev, const void* gate_dev, int32_t gstride,
                       int32_t goff, int32_t gstep, void* out_dev, int32_t l, int32_t p, int32_t lt, int32_t hq, int32_t hk,
                       int32_t hd, int32_t splits, void* ws_dev, size_t ws_bytes, void* stream);

/* `Gdn::subgroups` (`src/kernels.rs:257-302`): the gated delta rule over `batch` sequences of l tokens.
 * q_dev/k_dev [batch][l][qk_stride] (head h at h * 128), v_dev [batch][l][v_stride] (head h at h * 128),
 * f32, or f16 when in_f16; seq_qk/seq_v: elements between sequences. beta_dev and g_dev (the log decay:
 * the decay is exp(g)) [batch][l][h] f32; state_dev [batch][h][128][128] f32 (read when load_state,
 * always written); o_dev [batch][l][h * 128] f32. algo 0: the chunked scan (64-token chunks, one
 * pass; with f16 inputs the fused tcgen05 kernel, which needs 16-byte aligned q/k/v and strides of
 * multiples of 8 elements); 1: the token-serial recurrence (f32, batch 1); 2: the two-phase chunked
 * scan (f16, batch 1; needs scratch_dev of sd_gdn_scratch_bytes(l, h) bytes); 3: the single-pass
 * chunked scan on mma.sync (f16). */
int sd_gdn(const void* q_dev, const void* k_dev, int32_t qk_stride, const void* v_dev, int32_t v_stride,
           const void* beta_dev, const void* g_dev, void* state_dev, int32_t load_state, void* o_dev, int32_t l,
           int32_t h, int32_t batch, int64_t seq_qk, int64_t seq_v, int32_t in_f16, int32_t algo, void* scratch_dev,
           size_t scratch_bytes, void* stream);
size_t sd_gdn_scratch_bytes(int32_t l, int32_t h);

/* The two-phase scan of sd_gdn (algo 2: one sequence, f16 q/k/v) for callers that must not allocate
 * device memory while they run, such as a serving process whose GPU memory is all reserved when it
 * starts, or a latency path that cannot take cudaMalloc's implicit device synchronisation. This entry
 * point has no counterpart in the reference. It calls no cudaMalloc, cudaFree or other allocating
 * routine: its per-chunk scratch is one fixed 24 MiB device array inside the library. CUDA loads the
 * library's modules lazily, so a device commits those 24 MiB, and the library looks the array's
 * address up for it, when the gated-delta module first loads there: at sd_engine_create on that
 * device, or else at the first sd_gdn or sd_gdn_noalloc call on it. Make one of these happen at
 * start-up, before the process reserves the rest of its GPU memory and before any stream capture;
 * the device then holds the array until the process exits. Limit: ceil(l / 64) * h chunk records
 * must fit that array (sd_gdn_noalloc_max_tokens(h) tokens; 1088 for 16 heads); larger calls fail
 * with SD_ERR_INVALID and say why. All calls on a device share the array, and each call writes
 * every record it reads, so nothing carries over between calls; two calls whose work overlaps on
 * the GPU (different streams, no ordering between them) race on it. */
int sd_gdn_noalloc(const void* q_dev, const void* k_dev, int32_t qk_stride, const void* v_dev, int32_t v_stride,
                   const void* beta_dev, const void* g_dev, void* state_dev, int32_t load_state, void* o_dev, int32_t l,
                   int32_t h, void* stream);
/* The longest sequence sd_gdn_noalloc accepts for h heads. */
int32_t sd_gdn_noalloc_max_tokens(int32_t h);

/* A block-quantized int4 group-32 symmetric weight (`src/kernels.rs:545-576`) in the GEMM's tile
 * layout, made from the reference layout on the device: q_dev [n][k/32][16 bytes], s_dev [n][k/32] f16.
 * `interleave` stores rows (j, n/2 + j) next to each other (gate_up for the fused SwiGLU). */
int sd_qweight_create(const void* q_dev, const void* s_dev, int32_t n, int32_t k, int32_t interleave, sd_qweight** out);
/* sd_qweight_create for the reference's other formats (`src/kernels.rs:545-586`, served there by
 * `matmul_gemv`): bits 2, 3 or 4 (q_dev [n][k/32][4 * bits bytes]: int4 as 4 words of 8 nibbles, int2 as 2
 * words of 16 two-bit fields, int3 as those 2 words plus a word of high bits), one f16 scale per `group`
 * weights (a multiple of 32) indexed by the global block (row * k/32 + block) / (group / 32). b_dev null:
 * symmetric, value (q - 2^(bits-1)) * scale; else one f16 bias per group, indexed as the scales:
 * asymmetric, value q * scale + bias. The weight is repacked into the int4 tile layout with the same
 * values (the dequantized weight is rounded to f16 as the tiled path rounds it; the reference's
 * `matmul_gemv` keeps it f32). */
int sd_qweight_create_format(const void* q_dev, const void* s_dev, const void* b_dev, int32_t n, int32_t k, int32_t bits,
                             int32_t group, int32_t interleave, sd_qweight** out);
void sd_qweight_free(sd_qweight* w);

/* `matmul_gemv`/`matmul_tiled`/`matmul_coop` (`src/kernels.rs:590-804`): y_dev[m][ldy] =
 * f16(act_dev[m][k] W^T) (silu = 1 on an interleaved weight: y = silu(gate) * up, [m][n/2]).
 * ws_dev/ws_bytes: f32 workspace for split-K, one m * n slice per split (splits are reduced to fit;
 * 0 bytes disables split-K). Results do not depend on the split count's summation order run to run. */
int sd_matmul(const sd_qweight* w, const void* act_dev, int32_t m, void* y_dev, int32_t ldy, int32_t silu, void* ws_dev,
              size_t ws_bytes, void* stream);

/* sd_matmul with the kernel chosen and the residual add: algo 0 is sd_matmul's choice (where k is a
 * multiple of 128, the small-M kernel up to 16 tokens, or up to 64 with n <= 4096; else the tcgen05
 * tiles), 1 the tcgen05 tiles,
 * 2 the small-M kernel (mma.sync on weights dequantized in registers, K split over a thread-block
 * cluster; up to 256 tokens, k a multiple of 128; SD_ERR_INVALID otherwise). With x_dev (f32 rows,
 * ldy floats apart, 16-byte aligned; no silu) the f16-rounded products are added into x instead of
 * stored to y (y_dev may then be null): `add_norm`'s residual add (src/kernels.rs:93-120) done by the
 * matmul, as the engine runs it. Results of one algo do not change run to run. */
int sd_matmul_ex(const sd_qweight* w, const void* act_dev, int32_t m, void* y_dev, int32_t ldy, int32_t silu, void* x_dev,
                 void* ws_dev, size_t ws_bytes, int32_t algo, void* stream);

/* The standalone calls (sd_gdn, sd_attention*, sd_matmul) return once their kernels are queued; a
 * kernel that gave up (one of its bounded waits ran out, 2 s) records an error code on the device
 * instead of faulting. sd_op_status synchronises `stream`, reads and clears those codes on the
 * current device and returns SD_ERR_KERNEL (message: which call, which code) if any was set, else
 * SD_OK. No counterpart in the reference (its kernels have no such waits). The engine's calls check
 * their own error word and need no sd_op_status. */
int sd_op_status(void* stream);

/* `decode_scales` (`src/model.rs:219-236`) on the device: src_dev holds n 4-byte row headers (m as
 * fp16 bits, j as u16) then n rows of g codes (`sign << 7 | k`); dst_dev gets [n][g] fp16 with
 * |scale| = fp16(f32(m 2^(-k j / 4096))), the power in f64 from a host table as the reference builds
 * it, so bit-identical to the host decode. Synchronous (the headers are read to size the table).
 * sd_engine_create uses the same kernels for the embedding's 8-bit scale codes (`embed_parts`,
 * `src/model.rs:260-283`) and for packed shards (`unpack_shard`, `src/model.rs:239-258`: a shard
 * whose manifest entry has `wire` and whose converted weights.<i>.bin is absent is read from its
 * `path` and unpacked on the device). */
int sd_decode_scales(const void* src_dev, int32_t n, int32_t g, void* dst_dev, void* stream);

#ifdef __cplusplus
}
#endif
#endif
