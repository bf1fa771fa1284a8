/*
 * kh_cuda.h — C ABI of libkhcuda.so, the CUDA executor of kleinhirn Plans on B200 (sm_100a).
 *
 * The library is the device half of a `CudaBackend` that implements kleinhirn's `Backend` /
 * `PlanRunner` interface (src/backend.ts:14-46) beside src/webgpu-backend.ts and
 * src/wasm-backend.ts. It consumes the unchanged execution Plan (src/plan/ir.ts:41-60),
 * serialised as JSON, and the weights of the src/weights.ts loader (TensorDesc,
 * src/weights.ts:7-17). A host binding (N-API addon for Node, ctypes for Python) wraps these
 * functions one to one; no torch or other framework type appears in any signature.
 *
 * Conventions
 * - Every function that can fail returns int status: KH_OK (0) or a KH_ERR_* code. The message
 *   of the last failure on the calling thread is kh_last_error(); a binding turns a non-zero
 *   status into a thrown error with that message (as answer() does for the WASM worker,
 *   src/wasm-backend.ts:48-51).
 * - A CUDA error during a run latches in the context: every later call on that context fails
 *   with KH_ERR_STATE and the first message (mirrors failIfBroken, src/device.ts:79-81).
 * - Buffers passed in are host memory owned by the caller and are copied before the call
 *   returns (the WASM host copies inputs the same way, src/plan/wasm.ts:409-440); output
 *   buffers are host memory owned by the caller.
 * - One call in flight per plan (EncoderModel.enqueue serialises calls, src/encoder.ts:265-269).
 *   Distinct plans of one context share the context's stream.
 */
#ifndef KH_CUDA_H
#define KH_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kh_ctx kh_ctx;
typedef struct kh_plan kh_plan;
typedef struct kh_bulk kh_bulk;

enum kh_status {
  KH_OK = 0,
  KH_ERR_ARG = 1,   /* bad argument: sizes, null pointers, unknown tensor */
  KH_ERR_PLAN = 2,  /* the plan cannot run here (Backend.check) */
  KH_ERR_CUDA = 3,  /* a CUDA call failed */
  KH_ERR_STATE = 4  /* an earlier CUDA error latched in the context */
};

enum kh_dtype { KH_F32 = 0, KH_F16 = 1 };

/* Message of the last failure on this thread ("" when none). */
const char* kh_last_error(void);

/* Opens a context on devices[0]; n_devices must be 1 (KH_ERR_ARG otherwise: a context drives one
 * device, and a host that uses several devices opens one context per device and drives each from
 * its own thread). Replaces the device half of loadBackend / loadGpu (src/backend.ts:75-89,
 * src/webgpu-backend.ts:53-108). */
int kh_init(const int* devices, int n_devices, kh_ctx** out);

/* Copies one weight tensor to the device: TensorDesc name, dtype (KH_F32 or KH_F16), shape
 * (src/weights.ts:7-17) and its bytes from a verified shard (fetchShardBytes,
 * src/weights.ts:150-173). One createBuffer + writeBuffer per tensor in the WebGPU loader
 * (src/webgpu-backend.ts:53-101). The word table (keepOnCpu) is not added: it stays on the
 * host, as in src/wasm-backend.ts:184. */
int kh_add_tensor(kh_ctx* ctx, const char* name, int dtype, const int64_t* shape, int ndim, const void* bytes,
                  size_t len);

/* The word table from the bytes of words.bin (WordsDesc src/words-format.ts:6-18): `rows` rows of
 * `row_bytes` bytes, each `width` values of dtype (KH_F32 / KH_F16) followed by its checksum word
 * (wordsView, src/words.ts). Becomes the device tensor `name` [rows, width] without the checksums,
 * for kh_bulk_set_word_table. The caller has verified the file (fetchWords checks its sha256).
 * The reference keeps this table on the host; beyond the reference interface. */
int kh_add_words(kh_ctx* ctx, const char* name, int dtype, int64_t rows, int64_t width, int64_t row_bytes,
                 const void* bytes, size_t len);

/* Backend.weightBytes (src/backend.ts:32-33): device bytes of the loaded weights. */
int64_t kh_weight_bytes(const kh_ctx* ctx);

/* Backend.check (src/backend.ts:34-35): KH_OK when the plan can run, KH_ERR_PLAN with the
 * reason otherwise. Allocates nothing (src/plan/check.ts:119-124 checks before allocating). */
int kh_check(kh_ctx* ctx, const char* plan_json, size_t len);

/* Backend.runner (src/backend.ts:36): device buffers, derived weights and the launch list of
 * one Plan (JSON of src/plan/ir.ts:41-60, buffer init blobs as base64 under "init_b64"). */
int kh_plan_create(kh_ctx* ctx, const char* plan_json, size_t len, kh_plan** out);

/* PlanRunner.length / batch / bytes and the output shape (Plan.output rows x cols). */
int kh_plan_info(const kh_plan* plan, int* length, int* batch, int* out_rows, int* out_cols, int64_t* bytes);

/* PlanRunner.upload (src/backend.ts:20, RunInput src/plan/executor.ts:25-32): word rows
 * [batch * length * embeddingSize] in the plan's storage type (f16 bits for f16 plans, f32
 * otherwise), mask f32 [batch * length], typeIds u32 [batch * length] (low 16 bits the type,
 * high 16 bits the position row) or null when the plan has no typeIds input. Shorter inputs
 * are accepted, as writeBuffer writes a prefix. */
int kh_upload(kh_plan* plan, const void* emb, size_t emb_bytes, const float* mask, size_t mask_len,
              const uint32_t* type_ids, size_t type_len);

/* The marker part of RunInput for GLiNER2 / Julia plans (src/plan/executor.ts:25-37 packedMarkers
 * and qtype; uploads :366-388; type rows :236-246). `packed`: 3 * markers u32 per sequence of the
 * plan's batch — marker row indices local to the sequence, the marker mask as f32 bits, the
 * groups. `qtypes`: the Julia type of each sequence, a row of the plan's rowSelect table (null or
 * fewer entries: type 0, as `qtype ?? 0`; ignored by plans without type rows). Needed once
 * before kh_run for plans with a markers
 * input ("plan needs packedMarkers"); a qtype outside the table is KH_ERR_ARG. */
int kh_upload_markers(kh_plan* plan, const uint32_t* packed, size_t packed_len, const int32_t* qtypes,
                      size_t n_qtypes);

/* PlanRunner.run (src/backend.ts:21-23): one forward over `rows` rows — the real rows of a
 * B = 1 call (1 <= rows <= length), or length * batch for a batch plan. Queues the work and
 * returns. From the second call with a given `rows` on, the launch list runs as one CUDA graph
 * captured on that call (up to 8 row counts per plan); KH_NO_GRAPHS in the environment when the
 * plan is created keeps every run eager. */
int kh_run(kh_plan* plan, int rows);

/* PlanRunner.readOutput (src/backend.ts:24, src/plan/executor.ts:398-408): blocks until the
 * run is done and writes out_rows * out_cols f32 values (f16 storage converted). */
int kh_read_output(kh_plan* plan, float* out, size_t n);

/* Layer capture, the parity tool of PlanRunner.run(seqLen, capture = true) / readCapture /
 * assertCapturable (src/backend.ts:21-26; src/plan/executor.ts:178-186, :232, :267-281,
 * :418-424). kh_capture_check: KH_OK when the plan can capture (f32, batch 1), else KH_ERR_ARG
 * with the reference's reason. kh_run_capture: one forward over the full bucket that also runs
 * each segment's captureOps and, after the segment, copies the first captureSlotBytes of each of
 * its capture buffers into that buffer's slot. kh_read_capture: blocks, then writes the
 * captureSlots * captureSlotBytes / 4 f32 values. */
int kh_capture_check(const kh_plan* plan);
int kh_run_capture(kh_plan* plan);
int kh_read_capture(kh_plan* plan, float* out, size_t n);

/* PlanRunner.destroy (src/backend.ts:27). Also destroys the plan's bulk handles that are still
 * open; their handles are invalid afterwards. */
void kh_plan_destroy(kh_plan* plan);

/* Backend.dispose (src/backend.ts:45). Also destroys the context's plans and bulk handles that
 * are still open; their handles are invalid afterwards (a binding marks them destroyed). */
void kh_destroy(kh_ctx* ctx);

/* Backend.info (src/backend.ts:44): JSON with device name, SM count, memory, weight bytes.
 * Returns the bytes needed including the terminating zero; writes at most `cap` bytes. */
size_t kh_info(const kh_ctx* ctx, char* buf, size_t cap);

/* The launch list of a plan as JSON (one entry per kernel launch of kh_run, with the plan ops
 * it covers), for profiles and tests. Same size convention as kh_info. */
size_t kh_plan_launches(const kh_plan* plan, char* buf, size_t cap);

/* Raw bytes of a plan buffer by id, written from / read into host memory: the CUDA counterpart
 * of WasmPlan.view (src/plan/wasm.ts:473-476, "a plan buffer as f32 (tests, debugging)").
 * Used by the per-op known-answer tests; a read waits for the context stream. */
int kh_plan_buffer_write(kh_plan* plan, const char* id, const void* bytes, size_t len);
int kh_plan_buffer_read(kh_plan* plan, const char* id, void* out, size_t len);

/* Per-launch device times in ms of one forward over `rows` rows (CUDA events around every
 * launch), the CUDA counterpart of the WASM op profile (src/plan/wasm.ts:451-471) and of the
 * WebGPU dispatch profile (src/plan/executor.ts:303-361). Writes min(n, launches) values. */
int kh_profile(kh_plan* plan, int rows, float* ms, size_t n);

/* ---- ragged bulk runs: many sequences per call, only the rows a text has ----
 * Replaces the batch path of EncoderModel.runIdsBatch (src/encoder.ts:461-474), which pads to
 * batch plans of at most 16 sequences at a 64-row stride (src/cache.ts:9-19, :81-83): here the
 * sequences of one call are packed back to back and no padding row is computed.
 * A bulk handle holds device room for `max_tokens` packed input rows and `max_seqs` sequences
 * of one plan; its forward runs in chunks of at most `chunk_tokens` rows through one set of
 * activation buffers. Every sequence has all its rows valid (mask 1) and at most
 * plan.length rows. */
int kh_bulk_create(kh_plan* plan, int64_t max_tokens, int max_seqs, int64_t chunk_tokens, kh_bulk** out);

/* The sequences of the next run: n lengths in [1, plan.length], sum <= max_tokens. */
int kh_bulk_set_lengths(kh_bulk* bulk, const int32_t* seq_lens, int n);

/* Packed inputs of the sequences set last: word rows [sum(len) * embeddingSize] in the plan's
 * storage type and, when the plan has a typeIds input, typeIds [sum(len)] (type in the low, the
 * position row in the high 16 bits); type_ids may be null otherwise. Host to device copy. */
int kh_bulk_upload(kh_bulk* bulk, const void* emb, size_t emb_bytes, const uint32_t* type_ids, size_t type_len);

/* Device-resident word table for bulk runs: tensor `name` (added with kh_add_tensor, shape
 * [vocab, embeddingSize]) is kept on the device and the rows of packed token ids are gathered
 * there (kh_bulk_upload_ids), instead of the host gathering word rows (wordRows,
 * src/encoder.ts:273-314) from the table the reference keeps on the host
 * (src/wasm-backend.ts:184). Beyond the reference interface. */
int kh_bulk_set_word_table(kh_bulk* bulk, const char* name);

/* Packed token ids [sum(len)] int32 of the sequences set last, and typeIds as for
 * kh_bulk_upload (null when the plan has none); the word rows are gathered on the device. An id
 * outside [0, vocab) gives a zero row, and the next kh_bulk_read returns KH_ERR_ARG. */
int kh_bulk_upload_ids(kh_bulk* bulk, const int32_t* ids, size_t n, const uint32_t* type_ids, size_t type_len);

/* Device-side forward of every sequence (no host copies; returns when the launches are queued).
 * A run whose chunks have exactly the previous run's launch parameters (the same lengths
 * uploaded again) is captured as a CUDA graph on its second occurrence and replayed after;
 * KH_NO_GRAPHS in the environment when the handle is created keeps every run eager. */
int kh_bulk_run(kh_bulk* bulk);

/* Waits for the run and writes the outputs: one row of out_cols f32 per sequence for pooled
 * heads (n_seqs * out_cols values), one per packed row for token heads (sum(len) * out_cols). */
int kh_bulk_read(kh_bulk* bulk, float* out, size_t n);

/* set_lengths + upload + run + read in one call. */
int kh_run_batch(kh_bulk* bulk, const int32_t* seq_lens, int n, const void* emb, size_t emb_bytes,
                 const uint32_t* type_ids, size_t type_len, float* out, size_t out_len);

/* Device time in ms of the last kh_bulk_run (CUDA events on the context stream), and the
 * number of kernel launches it made. */
int kh_bulk_last_timing(const kh_bulk* bulk, float* ms, int64_t* launches);

/* Per-step device times in ms of one bulk forward, summed over its chunks (CUDA events around
 * every launch; one value per entry of kh_plan_launches). Not for timing runs: the events
 * serialise the launches. */
int kh_bulk_profile(kh_bulk* bulk, float* ms, size_t n);

/* Frees a bulk handle (kh_plan_destroy and kh_destroy free the ones still open). */
void kh_bulk_destroy(kh_bulk* bulk);

/* The CUDA stream (cudaStream_t) every launch of this context goes to, so a caller can record
 * its own events on it. The context owns the stream. */
void* kh_ctx_stream(const kh_ctx* ctx);

/* ---- allocation-free attention (no counterpart in the reference) ----
 * Packed multi-head attention of f16 plans, what the attention ops of a standard-attention plan
 * compute (src/kernels/attsoftmax.wgsl, mbattention.wgsl): per head softmax(scale q k^T) v over
 * the rows of the same sequence, masked keys and keys outside +-window (0: no window) left out,
 * masked query rows exactly zero. Caller-owned device buffers: qkv [T][3 * heads * head_dim]
 * f16 (the q, k and v blocks of each row, as the plan's qkv buffer), mask [T] f32 (1 keep,
 * 0 masked), ctx [T][heads * head_dim] f16 output; the T packed rows hold n_seqs sequences back
 * to back, T = the sum of seq_lens (host memory).
 *
 * It allocates no device memory, on any call: its sequence table lives in a static device array
 * of 563,200 bytes inside the library. It is for callers that cannot allocate at call time: a
 * serving loop whose device memory is budgeted up front, or code that must not let a cudaMalloc
 * synchronize the device in the middle of its work.
 * Limits: n_seqs <= 4096, T <= 65,536, each length in [1, 10,176], head_dim 32 or 64, qkv and
 * ctx 16-byte aligned; beyond them it returns KH_ERR_ARG and says which limit.
 * The first call on a device does one-time set-up (looks up the static array, sets the kernel's
 * shared-memory limit): make that call before any stream capture. All calls on a device share
 * the static array: calls that overlap in time (other streams, other host threads) race on it,
 * so the caller serializes them. The work is queued on `stream` (a cudaStream_t of the current
 * device, NULL for the legacy default stream; a stream of another device is KH_ERR_ARG); the
 * call returns once it is queued. seq_lens is read by a cudaMemcpyAsync on `stream`: from
 * pageable host memory it has been read when the call returns, from page-locked memory it is
 * read when the stream reaches the copy, so keep it unchanged until then.
 * A wait of the kernel's pipeline that gives up (a lost arrival, after 2 s) ends the kernel early
 * with ctx partly written and leaves a code on the device that this call cannot see, as the
 * kernel runs after it returns: kh_attention_f16_noalloc_status reports it. */
int kh_attention_f16_noalloc(const void* qkv, const float* mask, void* ctx, const int32_t* seq_lens, int n_seqs,
                             int heads, int head_dim, float scale, int window, void* stream);

/* Waits for `stream` (as cudaStreamSynchronize) and reports whether an attention kernel on the
 * current device gave up a pipeline wait since the last report: KH_OK, or KH_ERR_CUDA with the
 * wait's code. Reading clears the code. Callers of kh_attention_f16_noalloc check it before they
 * use ctx. (No counterpart in the reference.) */
int kh_attention_f16_noalloc_status(void* stream);

/* ---- failure-path self-tests (no counterpart in the reference) ----
 * They make the failure on purpose, in the forms that leave the GPU usable, so the error
 * handling of a context can be tested on a live device.
 * kh_inject_cuda_error: the next entry point of ctx that latches errors reports a CUDA failure
 *   named `what` (as if one of its CUDA calls had failed) and latches it, as failIfBroken does
 *   (src/device.ts:79-81): every later call on ctx then fails with KH_ERR_STATE.
 * kh_selftest_wait_limit: one CTA waits on an mbarrier nothing arrives on, with a limit of
 *   limit_us microseconds (1 to 1e6); the wait gives up and records its code as a pipeline wait
 *   that timed out does; the call synchronizes, returns KH_ERR_CUDA ("pipeline wait timed out")
 *   and latches it in ctx.
 * kh_selftest_tensor_maps: `threads` host threads (1-64) fetch `iters` TMA descriptors each from
 *   the library's descriptor cache over more keys than it keeps; returns how many differ from a
 *   fresh encoding (0 expected), or -1 on an error. */
int kh_inject_cuda_error(kh_ctx* ctx, const char* what);
int kh_selftest_wait_limit(kh_ctx* ctx, int limit_us);
int64_t kh_selftest_tensor_maps(int threads, int iters);

#ifdef __cplusplus
}
#endif

#endif /* KH_CUDA_H */
