/*
 * hawkb200.h -- C ABI of libhawkb200.so, the B200 (sm_100a) decoder engine.
 *
 * Drop-in replacement for the device side of the reference's single-dispatch
 * decoder engine (c8dhjp4tyv-bit/hawkpoint-npu-llm): the IRON designs
 * npu_llm/designs/{engine,qwen_engine}.py, their AIE2 kernels
 * npu_llm/kernels/{engine_bf16,qwen_engine_bf16,qwen_engine_hub_bf16}.cc, and the
 * host engines npu_llm/runtime/{engine,qwen_engine}.py.  Python binds it with
 * ctypes (hawkpoint-npu-llm_b200/runtime/hb_lib.py).
 *
 * Rules: every function returns 0 (HB_OK) or a negative HB_ERR_* code; the
 * message of the last failure is in hb_last_error().  An engine is not
 * thread-safe (one engine per GPU per process, calls serialised by the caller,
 * as npu_llm/api_server.py:646-678 serialises NPU calls).  The engine owns its
 * device memory; the caller owns host buffers.  Pointers named *_dev are device
 * pointers; all others are host pointers.  Device-side waits are bounded in
 * time; a wait that runs out makes the call return HB_ERR_DEVICE_TIMEOUT and
 * leaves the engine usable.  Every argmax follows np.argmax's order (a NaN
 * ranks above every number, the lowest index wins ties), so NaN logits select
 * the first NaN row as npu_llm/runtime/generate.py:713 does; a device-chained
 * token outside the vocabulary stops the chain with HB_ERR_STATE.
 */
#ifndef HAWKB200_H
#define HAWKB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HB_ABI_VERSION 1

enum {
  HB_OK = 0,
  HB_ERR_INVALID_ARG = -1,     /* bad argument: ValueError on the Python side */
  HB_ERR_CUDA = -2,            /* CUDA runtime error */
  HB_ERR_DEVICE_TIMEOUT = -3,  /* a bounded device wait gave up */
  HB_ERR_UNSUPPORTED = -4,     /* shape / layout this build does not run */
  HB_ERR_STATE = -5            /* e.g. weights not loaded */
};

enum { HB_FAMILY_LLAMA = 0, HB_FAMILY_QWEN2 = 1 };
enum { HB_WEIGHTS_BF16 = 0, HB_WEIGHTS_W8 = 1 };

/* hb_step / hb_prefill / hb_step_batch flags */
enum {
  HB_STEP_ARGMAX = 1,         /* run final norm + LM head + argmax */
  HB_STEP_LOGITS = 2,         /* also copy the FP32 logits out (implies ARGMAX) */
  HB_STEP_DEVICE_LOGITS = 4   /* keep the FP32 logits on the device for hb_sample
                                 (implies ARGMAX; no copy to the host) */
};

/* Byte offsets (from the start of the weight blob) of one layer's tensors.
 * The blob layout is defined by runtime/layout.py; the engine only validates
 * it.  Projections are stored "row-group major": 8 consecutive output rows
 * form a group, and a group stores its K dimension as 16-byte column chunks,
 * each chunk holding those 8 rows (chunk j of row r at group_base + j*128 +
 * r*16).  gate_up alternates 8 gate rows and the 8 matching up rows.  W8
 * projections store int8 in the same arrangement plus one FP32 scale per
 * (packed) row. */
typedef struct hb_layer_offsets {
  uint64_t gamma_in, gamma_post, qkv_bias;      /* FP32 [hidden], [hidden], [qkv] */
  uint64_t w_qkv, s_qkv;                        /* s_*: W8 row scales, else 0 */
  uint64_t w_o, s_o;
  uint64_t w_gate_up, s_gate_up;
  uint64_t w_down, s_down;
} hb_layer_offsets;

/* context: cache positions per slot.  <= 64 matches the reference's fixed
 * cache (npu_llm/runtime/generate.py:43-44).  A multiple of 64 up to 4096
 * (no reference counterpart) selects the paged cache: 64-position pages
 * behind a per-slot page table, pages zero-filled when first mapped,
 * hb_copy_prefix sharing whole pages that a slot copies only when it
 * writes into one, and the attention of long histories split over several
 * SMs.  Other values are HB_ERR_UNSUPPORTED. */
typedef struct hb_model_desc {
  int32_t abi_version;      /* HB_ABI_VERSION */
  int32_t family;           /* HB_FAMILY_* */
  int32_t hidden, intermediate, q_heads, kv_heads, head_dim, layers, vocab, context;
  int32_t has_qkv_bias;
  int32_t weight_format;    /* HB_WEIGHTS_* */
  int32_t max_slots;        /* independent KV-cache slots (streams) */
  int32_t max_batch;        /* rows per batched step (1 or 8) */
  float rms_eps;
  int32_t reserved0;
  uint64_t blob_bytes;
  uint64_t gamma_final, w_lm, s_lm, embedding;  /* embedding: BF16 row-major [vocab x hidden] */
  const hb_layer_offsets *layer_offsets;        /* [layers], host memory, copied */
  const float *rope_cos;    /* [context x head_dim/2], host memory, copied */
  const float *rope_sin;
} hb_model_desc;

typedef struct hb_engine hb_engine;

/* Engine lifecycle.  Replaces QwenDecoderEngine.__init__ / DecoderEngine.__init__
 * (npu_llm/runtime/qwen_engine.py:41-63, npu_llm/runtime/engine.py:32-49):
 * allocates the device weights, the KV cache of every slot and the step
 * buffers on `device`. */
int hb_create(const hb_model_desc *desc, int device, hb_engine **out);

/* Copies the packed weight blob (runtime/layout.py) to the device.  Replaces
 * the iron.tensor(pack_weights(...)) upload (npu_llm/runtime/qwen_engine.py:52-54). */
int hb_load_weights(hb_engine *engine, const void *host_blob, size_t bytes,
                    int layout_version);

/* Releases every device buffer.  Replaces QwenDecoderEngine.close
 * (npu_llm/runtime/qwen_engine.py:96-102).  Accepts NULL. */
int hb_destroy(hb_engine *engine);

/* One position of one stream through every layer, then (flags) the final
 * norm, the LM head and the argmax.  Replaces QwenDecoderEngine.step /
 * DecoderEngine.step (npu_llm/runtime/qwen_engine.py:77-94,
 * npu_llm/runtime/engine.py:65-82) plus the host argmax of
 * NPUDecoder._decode_result (npu_llm/runtime/generate.py:709-714).  The
 * embedding gather, RoPE and the K/V append all run on the device.
 * logits_out (host, [vocab] FP32) may be NULL; argmax_out may be NULL. */
int hb_step(hb_engine *engine, int slot, int token_id, int position, int flags,
            float *logits_out, int32_t *argmax_out);

/* Prefill of n prompt positions start_pos..start_pos+n-1, only the last
 * with the LM head -- the loop of npu_llm/runtime/generate.py:1110-1126.
 * With max_batch > 1 the positions before the last run up to 8 per launch
 * (same KV cache and result as one position per launch).  last_logits may
 * be NULL. */
int hb_prefill(hb_engine *engine, int slot, const int32_t *ids, int n,
               int start_pos, float *last_logits, int32_t *argmax_out);

/* Device-resident greedy generation (no host round trip per token): prefill
 * ids[start_pos..n_prompt-1], then n_new-1 further greedy steps feeding each
 * argmax back on the device.  out_tokens receives n_new ids.  Same result as
 * the host loop of npu_llm/runtime/generate.py:1110-1158 with greedy
 * selection and no stop strings. */
int hb_generate(hb_engine *engine, int slot, const int32_t *ids, int n_prompt,
                int start_pos, int n_new, int32_t *out_tokens);

/* Several streams, one position each, in one pass over the weights
 * (n <= max_batch).  New in this build (the reference serialises requests). */
int hb_step_batch(hb_engine *engine, int n, const int32_t *slots,
                  const int32_t *token_ids, const int32_t *positions, int flags,
                  float *logits_out, int32_t *argmax_out);

/* KV-cache management.  hb_reset replaces QwenDecoderEngine.reset
 * (npu_llm/runtime/qwen_engine.py:65-66); hb_copy_prefix copies positions
 * [0, n_positions) of every layer from one slot to another (prefix sharing).
 * With a paged cache (context > 64) hb_reset returns the slot's pages to the
 * pool, and hb_copy_prefix maps the source's whole pages below n_positions
 * into the destination (a page is copied when either slot next writes into
 * it) and copies the rows of a partial last page; the results are the same
 * as copying. */
int hb_reset(hb_engine *engine, int slot);
int hb_copy_prefix(hb_engine *engine, int src_slot, int dst_slot, int n_positions);

/* Diagnostics.  hb_debug_dump copies engine state for parity tests:
 * HB_DUMP_HIDDEN = BF16 residual stream [8 x hidden] after the last step;
 * HB_DUMP_KV = BF16 cache of one slot (paged: gathered from its pages, zeros
 * where none is mapped), per (layer, kv head) K then V, each
 * [context][head_dim] with the eight 16-byte blocks of a position stored at
 * block ^ (position & 7) (slot taken from *(int*)out on entry); HB_DUMP_TRACE = uint64 [SMs][4*layers+2][8] device timestamps of
 * the last launch traced with hb_profile(engine, 2). */
enum { HB_DUMP_HIDDEN = 0, HB_DUMP_KV = 1, HB_DUMP_TRACE = 2 };
const char *hb_last_error(const hb_engine *engine);
int hb_debug_dump(hb_engine *engine, int what, void *out, size_t bytes);

/* Profiling: when enabled (bit 0), each decode-kernel launch is bracketed by
 * CUDA events on the engine's stream; bit 1 also records per-phase device
 * timestamps of every CTA (hb_debug_dump kind 2).  hb_profile_read returns
 * the durations (ms) of up to max launches since the last read, and when
 * start_ms is not NULL each launch's start relative to the first one, then
 * clears the record. */
int hb_profile(hb_engine *engine, int enable);
int hb_profile_read(hb_engine *engine, float *ms, float *start_ms, int max, int *count);

/* Runs the engine's work on the caller's stream (cudaStream_t as void*);
 * NULL restores the engine's own stream. */
int hb_set_stream(hb_engine *engine, void *stream);

/* Fault-path test hook: the next launch makes every CTA wait on a device flag
 * that nothing sets, with the given limit (ns), so the bounded wait runs out
 * and the call returns HB_ERR_DEVICE_TIMEOUT.  No GPU fault is involved. */
int hb_test_stall_next(hb_engine *engine, uint64_t limit_ns);
/* The same for the next hb_gemv / hb_gemv_noalloc launch in the process: its
 * first CTA waits on a flag nothing sets until the limit passes, the launch
 * aborts, and the fused argmax of every batch row reads -1 (how both entry
 * points report a device wait that gave up; hb_gemv's scratch also holds the
 * timeout in its control block). */
int hb_test_gemv_stall_next(uint64_t limit_ns);

/* Standalone weight-streaming GEMV (the microbenchmark of the reference's
 * q_gemv4 / q_gemv_slice, npu_llm/kernels/qwen_engine_common.h:89-110, and
 * the BF16 projection of npu_llm/runtime/cpu_backend.py:64-69):
 *   y[b][r] = bf16(sum_k W[r][k] * x[b][k])        (HB_GEMV_OUT_BF16)
 *   y[b][r] = sum_k W[r][k] * x[b][k]   (FP32)     (HB_GEMV_OUT_F32)
 * with W8 weights the sum is multiplied by scales[r] before rounding.
 * HB_GEMV_ARGMAX also writes argmax_dev[b] (first index of the maximum, as
 * np.argmax).  W is packed row-group major (runtime/layout.py); rows % 8 == 0,
 * k % 32 == 0; batch is 1..8.  All pointers are device pointers; scratch_dev
 * must hold hb_gemv_scratch_bytes(rows, batch) bytes.  Runs on `stream`.
 * If a bounded device wait gives up, every argmax_dev[b] reads -1 and the
 * control block at the start of scratch_dev records the timeout. */
enum { HB_GEMV_OUT_BF16 = 0, HB_GEMV_OUT_F32 = 1, HB_GEMV_OUT_NONE = 2 };
enum { HB_GEMV_ARGMAX = 4 };
size_t hb_gemv_scratch_bytes(int rows, int batch);
int hb_gemv(const void *w_dev, const float *scales_dev, int weight_format,
            int rows, int k, const void *x_dev, int batch, void *y_dev,
            int flags, int32_t *argmax_dev, void *scratch_dev,
            size_t scratch_bytes, void *stream);

/* hb_gemv without the scratch argument, for callers that cannot allocate
 * device memory -- e.g. a serving process whose GPU memory pool was sized at
 * start-up and forbids later allocations, or a hot path that must not call
 * cudaMalloc/cudaFree because they can synchronize the device.  No
 * counterpart in the reference (its NPU path has no device allocator).
 * Same arguments and results as hb_gemv; the scratch is a fixed 65,568-byte
 * __device__ array inside the library (room for batch <= 8 and up to 1024
 * CTAs; larger requests return HB_ERR_UNSUPPORTED), held by every GPU that
 * loads the library until the process exits.  The first call on a device
 * looks the array's address up (make it before any stream capture) and
 * keeps it for the primary context, so do not call it again after a
 * cudaDeviceReset.  All calls on a device share the array: calls that may
 * overlap on the GPU (unordered streams) race.  A device wait that gives up
 * shows as argmax_dev[b] == -1 for every row (the control block is inside
 * the library).  Allocates nothing; errors in hb_library_error(). */
int hb_gemv_noalloc(const void *w_dev, const float *scales_dev, int weight_format,
                    int rows, int k, const void *x_dev, int batch, void *y_dev,
                    int flags, int32_t *argmax_dev, void *stream);

/* ---- token sampling on the device -------------------------------------
 * The selection of the reference's Sampler.select
 * (npu_llm/runtime/sampling.py:416-445, which the host runs on a logits copy
 * at npu_llm/runtime/generate.py:1070-1080): penalties over the history,
 * logit bias, temperature (0 = argmax), top-k, top-p and the multinomial
 * draw, in that order and with NumPy's FP32/FP64 rounding and summation
 * order.  The one random number the draw consumes, `uniform`, is the
 * request generator's next Generator.random() on the host (what
 * Generator.choice would consume), so a seeded request keeps its stream.
 * history_* are the unique in-vocabulary history tokens and their counts
 * (np.unique of the history, as sampling.py:346-353 computes them); bias_*
 * the in-vocabulary logit_bias entries, each token once.  Parameters that
 * cannot reorder the logits (the reference's `greedy`) select the argmax
 * and ignore `uniform`.  Returns HB_ERR_UNSUPPORTED (token -1) when top_p
 * keeps more than 4096 candidates -- the caller then selects on the host;
 * HB_ERR_INVALID_ARG for out-of-range parameters or ids.  Vocabularies up
 * to 262,144 entries. */
typedef struct {
  float temperature, top_p, repetition_penalty, presence_penalty, frequency_penalty;
  int32_t top_k;
  int32_t n_history;
  const int32_t *history_tokens;
  const float *history_counts;
  int32_t n_bias;
  const int32_t *bias_tokens;
  const float *bias_values;
  double uniform;
} hb_sampling;

typedef struct hb_sampler hb_sampler;
/* A standalone sampler for `vocab`-wide logits on `device` (owns its device
 * scratch and its stream).  Vocabularies of 16,384 and more select with one
 * thread block per SM (a cooperative launch), smaller ones with one. */
int hb_sampler_create(int vocab, int device, hb_sampler **out);
/* Select from `logits` (host memory, or device memory when
 * logits_on_device is nonzero). */
int hb_sampler_select(hb_sampler *sampler, const float *logits, int logits_on_device,
                      const hb_sampling *params, int32_t *token_out);
int hb_sampler_destroy(hb_sampler *sampler);
/* Log-probabilities of an OpenAI `logprobs` entry from the raw logits: the
 * reference's float64 log_softmax (npu_llm/runtime/stopping.py:101-109) at
 * `token`, and the n_top (<= 32) largest entries in descending order (equal
 * scores by index descending) as npu_llm/runtime/generate.py builds them
 * with np.argpartition + argsort.  Differences from NumPy: the float64 exp
 * and log of CUDA against the host libm (an ulp). */
int hb_sampler_logprobs(hb_sampler *sampler, const float *logits, int logits_on_device, int token,
                        int n_top, double *token_logprob, int32_t *top_ids, double *top_logprobs);
/* Select from row `row` of the logits the engine's last hb_step /
 * hb_step_batch left on the device (HB_STEP_DEVICE_LOGITS), on the
 * engine's stream. */
int hb_sample(hb_engine *engine, int row, const hb_sampling *params, int32_t *token_out);
/* Several selections in one launch (one thread block each), for a batched
 * step (hb_step_batch with HB_STEP_DEVICE_LOGITS): entry k selects from
 * logits row rows[k] with params[k].  tokens_out[k] = -1 marks an entry
 * whose top-p nucleus is too large for the device (select it on the host
 * from hb_read_logits).  n <= max_batch.  New in this build (the reference
 * serves one request at a time). */
int hb_sample_batch(hb_engine *engine, int n, const int32_t *rows, const hb_sampling *params,
                    int32_t *tokens_out);
/* hb_sampler_logprobs on row `row` of the engine's device logits. */
int hb_logprobs(hb_engine *engine, int row, int token, int n_top, double *token_logprob,
                int32_t *top_ids, double *top_logprobs);
/* Copy rows [0, n_rows) of the FP32 logits the last step left on the device
 * to logits_out (host, n_rows x vocab) -- the host-selection fallback after
 * hb_sample returned HB_ERR_UNSUPPORTED, without recomputing the step. */
int hb_read_logits(hb_engine *engine, int n_rows, float *logits_out);

/* ---- tensor-core GEMM for batched rows (new in this build) ------------------
 * y[n][r] = sum_k W[r][k] * X[n][k] on the 5th-generation tensor cores
 * (tcgen05.mma, BF16 inputs, FP32 accumulate in tensor memory): the dense
 * contraction that batched prefill and multi-stream decode reduce to.  The
 * reference runs these projections one position at a time
 * (npu_llm/runtime/generate.py:1110-1126, one engine dispatch per position;
 * npu_llm/designs/qwen_engine.py:158-212 inside the dispatch).
 * w_dev: BF16 rows x k in the packed row-group layout (runtime/layout.py
 * pack_matrix_bytes); x_dev: BF16 n x k activations in the same layout, n
 * rounded up to a multiple of 8 rows; y_dev: FP32 [n][rows].  rows a
 * multiple of 8, k of 64, 1 <= n <= 256, operands 16-byte aligned.  The
 * caller owns scratch_dev (hb_tc_gemm_scratch_bytes: the control block;
 * split-K partial sums stay in the cluster's shared memory); each call
 * clears it, so calls on one scratch must not overlap.
 * Asynchronous on `stream`; hb_tc_gemm_status() waits for the stream and
 * reports a device-side wait that gave up. */
size_t hb_tc_gemm_scratch_bytes(int rows, int k, int n);
int hb_tc_gemm(const void *w_dev, int rows, int k, const void *x_dev, int n, float *y_dev, void *scratch_dev,
               size_t scratch_bytes, void *stream);
int hb_tc_gemm_status(const void *scratch_dev, void *stream);

/* ---- batched step on the tensor cores (new in this build) -------------------
 * n rows (1 <= n <= 256) through every layer, the final norm and the LM
 * head in one call: row i feeds token_ids[i] at positions[i] of KV slot
 * slots[i].  The final norm and LM head run over the output rows only: with
 * out_rows NULL (n_out == n) every row, else the n_out rows out_rows[0..)
 * (e.g. the last position of each sequence in a chunked-prefill step).
 * Output j's argmax goes to argmax_out[j] and, when logits_out is not NULL,
 * its FP32 logits to logits_out[j * vocab ...].  Rows may mix
 * sequences (multi-stream decode) and may hold consecutive positions of one
 * sequence (chunked prefill): every row's K/V is appended before any row
 * attends, so a row sees the rows of its sequence at earlier positions.  No
 * two rows may write the same (slot, position).  Per layer: RMSNorm, qkv
 * (tcgen05 GEMM + bias), RoPE and K/V append, attention, o (GEMM +
 * residual), RMSNorm, gate/up (GEMM + SwiGLU), down (GEMM + residual), with
 * the reference's BF16 rounding points (npu_llm/runtime/cpu_backend.py:131-181);
 * FP32 sums run in a different order than the persistent kernel's, so
 * results agree with hb_step to the documented tolerance, not bit for bit.
 * BF16 weights and the 64-position cache only (HB_ERR_UNSUPPORTED otherwise).
 * Replaces the reference's one dispatch per position
 * (npu_llm/runtime/generate.py:1110-1126) and its single-lock serving
 * (npu_llm/api_server.py:646-678) for the rows it batches. */
int hb_step_rows(hb_engine *engine, int n, const int32_t *slots, const int32_t *token_ids,
                 const int32_t *positions, int n_out, const int32_t *out_rows, int32_t *argmax_out,
                 float *logits_out);
/* Prefill of positions start_pos .. start_pos + n - 1 of one slot through
 * hb_step_rows (256 rows per launch sequence, the LM head on each chunk's
 * last row only); the last position's argmax and, when last_logits is not
 * NULL, its FP32 logits. */
int hb_prefill_tc(hb_engine *engine, int slot, const int32_t *ids, int n, int start_pos, float *last_logits,
                  int32_t *argmax_out);

/* Library-level error text (for calls that have no engine, e.g. hb_gemv). */
const char *hb_library_error(void);

/* Number of multiprocessors the persistent kernels are sized for on `device`
 * (0 when no device is present). */
int hb_device_sm_count(int device);

#ifdef __cplusplus
}
#endif

#endif /* HAWKB200_H */
