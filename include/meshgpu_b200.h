/*
 * meshgpu_b200.h — C ABI of the B200 stage executor.
 *
 * One `mg_stage` is one pipeline stage of a dense decoder (Llama or Qwen3
 * architecture): an optional token embedding (first stage), a contiguous range
 * of decoder layers [layer_start, layer_end), and an optional final RMSNorm +
 * lm_head (last stage).  The stage owns its weights in HBM and a KV cache per
 * request slot.  Every pointer argument that names tensor data is a device
 * pointer on the stage's GPU unless the comment says "host".  All functions
 * return an `int` status (MG_OK on success) and never abort; the message of
 * the last failure on the calling thread is returned by `mg_last_error()`.
 *
 * Each entry point replaces a call of the reference's portable backend
 * (hungtrab/gpu_mesh, Python); the replaced interface is cited beside it.
 * Calls on one stage handle must be serialised by the caller (the Python
 * worker holds a re-entrant lock, as the reference's StageWorker does,
 * src/meshgpu/backends/portable/stage_worker.py:117-121).
 */
#ifndef MESHGPU_B200_H
#define MESHGPU_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  MG_EINVAL maps to the reference's ValueError cases
 * (shape / position / vocab / cache-layout violations), MG_ESTATE to its
 * RuntimeError cases (protocol state such as an empty or short cache). */
#define MG_OK 0
#define MG_EINVAL 1
#define MG_ESTATE 2
#define MG_ECUDA 3
#define MG_ENOMEM 4
#define MG_EDEVICE 5 /* a kernel recorded an out-of-range id or position */
#define MG_ETIMEOUT 6 /* a kernel gave up a bounded wait (about 2 s); its outputs are invalid */

#define MG_DTYPE_F32 0
#define MG_DTYPE_BF16 1

/* Output selection for mg_stage_forward on the last stage. */
#define MG_OUT_HIDDEN 0      /* non-last stage: hidden states [B,S,H]           */
#define MG_OUT_LOGITS_ALL 1  /* logits for every position [B,S,V] (reference)   */
#define MG_OUT_LOGITS_LAST 2 /* logits of the last position only [B,1,V]         */

/* Attention mask policy, mirroring LlamaStage.forward
 * (src/meshgpu/models/llama_dense.py:497-532). */
#define MG_ATTN_SDPA 0  /* S==1 decode attends to every cached key; else key j <= position */
#define MG_ATTN_EAGER 1 /* always key j <= position                                       */

typedef struct mg_stage mg_stage;

/* Model + stage geometry.  Replaces LlamaConfig (llama_dense.py:20-78) plus
 * the layer range and endpoint flags of LlamaStage.__init__
 * (llama_dense.py:301-348) and Qwen3Stage.__init__ (models/qwen3_hf.py:62-144). */
typedef struct mg_stage_config {
  int32_t vocab_size;
  int32_t hidden_size;
  int32_t intermediate_size;
  int32_t num_hidden_layers;
  int32_t num_attention_heads;
  int32_t num_key_value_heads;
  int32_t head_dim;
  int32_t max_position_embeddings;
  float rms_norm_eps;
  int32_t qk_norm;        /* 1 = Qwen3 per-head RMSNorm on q and k before RoPE */
  int32_t attention_impl; /* MG_ATTN_SDPA or MG_ATTN_EAGER */
  int32_t dtype;          /* MG_DTYPE_F32 or MG_DTYPE_BF16 */
  int32_t layer_start;
  int32_t layer_end;
  int32_t has_embedding;
  int32_t has_lm_head;
  int32_t device;         /* CUDA device ordinal */
} mg_stage_config;

/* Device pointers of one decoder layer, in the reference's nn.Linear layout
 * ([out_features, in_features], row-major).  q_norm / k_norm are NULL unless
 * qk_norm is set.  Names follow LlamaDecoderLayer (llama_dense.py:251-257) and
 * the HF Qwen3DecoderLayer state-dict keys. */
typedef struct mg_layer_weights {
  const void* input_layernorm;          /* [H] */
  const void* q_proj;                   /* [nq*D, H] */
  const void* k_proj;                   /* [nkv*D, H] */
  const void* v_proj;                   /* [nkv*D, H] */
  const void* q_norm;                   /* [D] or NULL */
  const void* k_norm;                   /* [D] or NULL */
  const void* o_proj;                   /* [H, nq*D] */
  const void* post_attention_layernorm; /* [H] */
  const void* gate_proj;                /* [I, H] */
  const void* up_proj;                  /* [I, H] */
  const void* down_proj;                /* [H, I] */
} mg_layer_weights;

/* Endpoint tensors.  embed_tokens is read when has_embedding; norm and lm_head
 * when has_lm_head (for tied embeddings pass the embedding matrix as lm_head).
 * rope_cos / rope_sin are the [max_position_embeddings, head_dim/2] tables in
 * the stage dtype, built with the reference's formula
 * (llama_dense.py:96-104, cast to the activation dtype as at :431-432). */
typedef struct mg_stage_weights {
  const void* embed_tokens; /* [V, H] or NULL */
  const void* norm;         /* [H] or NULL */
  const void* lm_head;      /* [V, H] or NULL */
  const void* rope_cos;     /* [max_pos, D/2] */
  const void* rope_sin;     /* [max_pos, D/2] */
  const mg_layer_weights* layers; /* host array of (layer_end - layer_start) entries */
} mg_stage_weights;

/* Library version string (host). */
const char* mg_version(void);

/* Message of the last failed call on this thread (host string, never NULL). */
const char* mg_last_error(void);

/* Build a stage: validates the geometry (LlamaConfig.__post_init__,
 * llama_dense.py:35-74; StageContext.__post_init__, stage_worker.py:45-63),
 * copies the weights into the stage's own HBM layout and returns a handle.
 * The caller may free its weight tensors afterwards.  Replaces
 * LlamaStage.__init__ + StageWorker.__init__ (llama_dense.py:301-348,
 * stage_worker.py:109-123) and the per-stage load of
 * build_stage_from_manifest (artifacts/hf_import.py:729-857). */
int mg_stage_create(const mg_stage_config* cfg, const mg_stage_weights* weights, mg_stage** out);

/* Release the stage, its weights and every KV slot. */
int mg_stage_destroy(mg_stage* stage);

/* Bytes of HBM held by the stage (weights + KV slots + work buffers). */
int mg_stage_memory(const mg_stage* stage, uint64_t* weight_bytes, uint64_t* kv_bytes,
                    uint64_t* work_bytes);

/* ---- KV slots: one per request context (cache_key).  Replace the named
 * cache dictionary of StageWorker (stage_worker.py:358-416). ---- */

/* Create (or re-create, dropping contents) slot `slot` for `batch` rows and
 * room for `capacity` positions.  A slot grows by itself when a forward would
 * overflow it, up to max_position_embeddings. */
int mg_kv_alloc(mg_stage* stage, int32_t slot, int32_t batch, int32_t capacity);

/* Drop a slot (StageWorker.clear_kv, stage_worker.py:369-375).  Dropping a
 * slot that does not exist is not an error. */
int mg_kv_free(mg_stage* stage, int32_t slot);

/* Drop every slot (StageWorker.clear_all_kv, stage_worker.py:377-381). */
int mg_kv_free_all(mg_stage* stage);

/* Cached length of a slot; 0 for an absent slot
 * (StageWorker.kv_cache_length, stage_worker.py:383-393). */
int mg_kv_length(const mg_stage* stage, int32_t slot, int32_t* length);

/* Batch rows of a slot; 0 for an absent slot. */
int mg_kv_batch(const mg_stage* stage, int32_t slot, int32_t* batch);

/* Trim a slot to `length` positions (StageWorker.trim_kv,
 * stage_worker.py:395-416): MG_EINVAL for a negative length, MG_ESTATE for an
 * absent slot with a non-zero length or a cache shorter than `length`. */
int mg_kv_trim(mg_stage* stage, int32_t slot, int32_t length);

/* Copy `length` positions of K and V for one local layer into a slot, which
 * must already hold `batch` rows.  `k` and `v` are [batch, nkv, length, D] in
 * the stage dtype (the layout of the reference's cache tuples,
 * llama_dense.py:166-170).  Sets the slot length to `length` once all layers
 * have been written; used to pre-fill long contexts. */
int mg_kv_import(mg_stage* stage, int32_t slot, int32_t local_layer, const void* k, const void* v,
                 int32_t length, void* stream);

/* Copy the cached K and V of one local layer out of a slot into
 * [batch, nkv, length, D] buffers (the reference's ForwardResult.kv_caches). */
int mg_kv_export(const mg_stage* stage, int32_t slot, int32_t local_layer, void* k, void* v,
                 void* stream);

/* ---- Weights in the stage's HBM arena ---- */

#define MG_W_EMBED 0      /* embed_tokens.weight [V, H] (first stage)                */
#define MG_W_NORM 1       /* norm.weight [H] (last stage)                             */
#define MG_W_LM_HEAD 2    /* lm_head.weight [V, H] (last stage; the embedding if tied) */
#define MG_W_INPUT_NORM 3 /* layers.i.input_layernorm.weight [H]                      */
#define MG_W_QKV 4        /* layers.i q_proj, k_proj, v_proj rows stacked [(nq+2nkv)D, H] */
#define MG_W_Q_NORM 5     /* layers.i.self_attn.q_norm.weight [D] (Qwen3)             */
#define MG_W_K_NORM 6     /* layers.i.self_attn.k_norm.weight [D] (Qwen3)             */
#define MG_W_O 7          /* layers.i.self_attn.o_proj.weight [H, nq D]               */
#define MG_W_POST_NORM 8  /* layers.i.post_attention_layernorm.weight [H]             */
#define MG_W_GATE_UP 9    /* layers.i gate_proj then up_proj rows [2I, H]             */
#define MG_W_DOWN 10      /* layers.i.mlp.down_proj.weight [H, I]                     */

/* Device address of one weight of the stage (row-major, the stage dtype;
 * NULL where the stage has no such weight).  The fused q/k/v and gate/up
 * matrices hold the reference's separate matrices as consecutive row blocks,
 * so each reference parameter is a contiguous slice.  Backs the stage's
 * named_parameters / state_dict / load_state_dict (LlamaStage is an
 * nn.Module, llama_dense.py:293; callers read named_parameters,
 * inference/server.py:458). */
int mg_stage_weight(const mg_stage* stage, int32_t which, int32_t local_layer, void** ptr);

/* ---- Forward ---- */

/* Run the stage for one request slot: embedding (first stage) or hidden
 * input, every local decoder layer, KV append at the slot's current length,
 * and on the last stage the final norm + lm_head.  Replaces
 * StageWorker.forward_inference (stage_worker.py:129-170) with
 * LlamaStage.forward (llama_dense.py:350-578) / Qwen3Stage.forward
 * (models/qwen3_hf.py:146-292).
 *   input_ids  int64 [batch, seq] (first stage) or NULL
 *   hidden_in  [batch, seq, H] in the stage dtype (other stages) or NULL
 *   positions  int64 [batch, seq], or NULL for arange(T, T+seq) with T the
 *              slot's cached length (llama_dense.py:482-491)
 *   out        hidden [batch, seq, H], or logits per out_mode
 * The slot is created for `batch` rows if absent; a present slot must hold
 * `batch` rows.  Kernels run on `stream` (a cudaStream_t, NULL = legacy). */
int mg_stage_forward(mg_stage* stage, int32_t slot, const int64_t* input_ids,
                     const void* hidden_in, const int64_t* positions, int32_t batch,
                     int32_t seq, int32_t out_mode, void* out, void* stream);

/* Single-token decode for several slots at once: rows of all slots are
 * stacked into one batch (slot order), every weight is streamed once for the
 * whole batch, and each row attends to its own slot's cache.  Equivalent to
 * one mg_stage_forward(seq=1, positions=NULL) per slot.  `slots` is a host
 * array; input/out are [sum(batch of slots), 1, ...]. */
int mg_stage_decode_multi(mg_stage* stage, const int32_t* slots, int32_t n_slots,
                          const int64_t* input_ids, const void* hidden_in, int32_t out_mode,
                          void* out, void* stream);

/* mg_stage_decode_multi on the last stage with the greedy token of every row
 * selected on the device: ids_out (device int64 [rows]) receives argmax of
 * the row's bf16/fp32 logits, the lowest index among equal maxima, as
 * greedy_sample (inference/sampling.py:45-56) on the logits the reference's
 * stage returns.  With the bf16 decode GEMM the selection is fused into the
 * lm_head epilogue; logits_out ([rows, 1, V]) may be NULL when the logits are
 * not wanted.  Replaces the per-step logits round trip of the reference's
 * decode loops (session.py:245-259, batcher.py:356-388). */
int mg_stage_decode_greedy(mg_stage* stage, const int32_t* slots, int32_t n_slots,
                           const int64_t* input_ids, const void* hidden_in, int64_t* ids_out,
                           void* logits_out, void* stream);

/* mg_stage_decode_multi on the last stage plus top_p_sample of every row
 * (inference/sampling.py:63-95) with temperature > 0: the lm_head's epilogue
 * counts each row's bf16 logits by value into a histogram, and one selection
 * kernel draws the token for uniforms[r] by the rule of mg_sample_top_p
 * (the same token, up to the rounding of the cumulative sums).  The logits
 * [rows, V] are also written to `logits_out` (the selection reads them).
 * fp32 stages sample the written logits with mg_sample_top_p's kernel. */
int mg_stage_decode_top_p(mg_stage* stage, const int32_t* slots, int32_t n_slots, const int64_t* input_ids,
                          const void* hidden_in, float temperature, float top_p, const float* uniforms,
                          int64_t* ids_out, void* logits_out, void* stream);

/* Read and clear the stage's device error word (waits for `stream`).
 * Returns MG_EDEVICE with a message when a kernel met an out-of-range token
 * id or position since the last check. */
int mg_stage_check_device(mg_stage* stage, void* stream);

/* Exercise the stage's timeout path without a fault: one thread waits, with
 * the same bounded wait every kernel of the stage uses, for a flag word of the
 * stage that is set only when `flag_set` is non-zero.  With the flag unset the
 * wait runs out after `limit_us` (1 .. 2e6) and records code 3 in the stage's
 * error word, exactly as a starved tensor-core kernel would; the next
 * mg_stage_check_device returns MG_ETIMEOUT and resets the stage's counters.
 * Nothing else is in flight during the wait.  Instrumentation; no
 * counterpart in the reference, which tests failures on the host only
 * (tests/unit/test_inference.py:196-233). */
int mg_stage_probe_wait(mg_stage* stage, uint32_t limit_us, int32_t flag_set, void* stream);

/* ---- Single linear layer (the stage's GEMM paths: weight-streaming GEMV
 * for <= 32 rows, tcgen05 GEMM above, SIMT for fp32) ---- */

#define MG_EPI_STORE 0  /* Y = round(X·Wᵀ)                                     */
#define MG_EPI_RESID 1  /* Y = round(R + round(X·Wᵀ))   (o_proj / down_proj)     */
#define MG_EPI_SWIGLU 2 /* W = [gate; up] ([2N, K]); Y = round(round(silu(round(g))) * round(u)) */

/* Y[M, N] = epilogue(X[M, K] · W[N, K]ᵀ) in `dtype`, the nn.Linear of the
 * reference (llama_dense.py:140-143, 239-244) with its rounding points.
 * `scratch` (fp32, `scratch_elems` elements) serves the split-K GEMV; the
 * bytes it needs are returned by mg_linear_scratch.  R may alias Y. */
int mg_linear(int32_t dtype, const void* X, int64_t ldx, const void* W, int32_t M, int32_t N,
              int32_t K, int32_t epilogue, const void* R, int64_t ldr, void* Y, int64_t ldy,
              float* scratch, uint64_t scratch_elems, void* stream);

/* fp32 scratch elements mg_linear needs for this shape. */
uint64_t mg_linear_scratch(int32_t dtype, int32_t M, int32_t N, int32_t K, int32_t epilogue);

/* Status of the mg_linear / mg_linear_noalloc launches on the current device
 * since the last check: waits for `stream`, then returns MG_EDEVICE if a
 * launch gave up waiting for its data (a bounded wait of about 2 s ran out;
 * that launch's Y is invalid), and clears the status.  The launches
 * themselves return as soon as they are queued, so they cannot report it.
 * Instrumentation of this library's own kernels; no counterpart in the
 * reference. */
int mg_linear_check_device(void* stream);

/* The same linear layer as mg_linear, for callers that cannot allocate
 * device memory: a process whose device memory is owned by another
 * allocator (a serving framework's caching allocator, say) and may not take
 * cudaMalloc / cudaFree behind it, or a latency-bound loop that cannot afford
 * the device-wide synchronisation those calls bring.  No counterpart in the
 * reference, which has no kernels of its own.
 *
 * It takes no scratch argument and allocates nothing: the split-K scratch of
 * the decode GEMV is one fixed array in the library (MG_LINEAR_NOALLOC_SCRATCH
 * fp32 elements, 4 MiB), present on every GPU that loads the library until
 * the process exits.  That covers the decode layers of the benchmark models
 * up to 16 token rows; a shape whose split-K needs more fails with MG_EINVAL
 * and says how much it needs.  Each call looks up the current device's copy of
 * the array (the lookup during a stream capture reuses the previous call's
 * address), so make one call per device before any stream capture.  A bounded
 * wait that runs out is reported by mg_linear_check_device.  All calls on one device within a process share the
 * array and leave their partial sums in it; the tile counters at its front
 * must start at zero, so every call clears them first (an asynchronous
 * memset on `stream`, no allocation).  Two calls that overlap on the GPU,
 * for example on two streams, race on the array, so serialise them. */
#define MG_LINEAR_NOALLOC_SCRATCH (1024u * 1024u)
int mg_linear_noalloc(int32_t dtype, const void* X, int64_t ldx, const void* W, int32_t M,
                      int32_t N, int32_t K, int32_t epilogue, const void* R, int64_t ldr, void* Y,
                      int64_t ldy, void* stream);

/* ---- Instrumentation (no counterpart in the reference, which has no
 * kernels of its own; used by the benchmark to report roofline fractions) ---- */

#define MG_PROF_LINEAR_DECODE 0  /* weight-streaming GEMV launches (<= 32 token rows) */
#define MG_PROF_LINEAR_PREFILL 1 /* GEMM launches (> 32 token rows) */
#define MG_PROF_ATTENTION 2      /* attention launches */
#define MG_PROF_OTHER 3          /* norms, RoPE/KV append, embedding, copies */
#define MG_PROF_CLASSES 4

typedef struct mg_profile {
  double ms[MG_PROF_CLASSES];          /* summed device time of the timed launches per class */
  double bytes[MG_PROF_CLASSES];       /* their algorithmic HBM bytes (operands read + written once) */
  double flops[MG_PROF_CLASSES];       /* their algorithmic FLOPs */
  uint64_t launches[MG_PROF_CLASSES];  /* launch groups timed */
} mg_profile;

/* Start (enable=1) or stop (0) timing every launch group of this stage with
 * CUDA events on its stream; starting resets the accumulated profile. */
int mg_stage_profile(mg_stage* stage, int32_t enable);

/* Wait for the timed launches and return the accumulated profile. */
int mg_stage_profile_read(mg_stage* stage, mg_profile* out);

/* Kernels launched by this library in this process so far. */
uint64_t mg_launch_count(void);

/* ---- Stage boundaries between GPUs of one process ----
 * Replace the reference's move_boundary / probe_cuda_path
 * (transport/local_cuda.py:27-90), which moves a stage output with
 * Tensor.to on the caller's stream: here the copy is queued on a side stream
 * of the caller's choosing, ordered by events, into a buffer the receiving
 * stage owns. */

/* Let `device` read and write `peer`'s memory over NVLink (every B200 pair on
 * an NVSwitch box).  *enabled = 1 if the pair has peer access (now enabled),
 * 0 if copies between them must stage through host memory. */
int mg_peer_access(int32_t device, int32_t peer, int32_t* enabled);

/* Leave `n` SMs of `device` (0 <= n <= half of them) out of the persistent
 * decode kernels' grids (the decode GEMM, decode and prefill attention), so
 * kernels that run beside them (NCCL's send/receive kernels in a
 * multi-process pipeline) never hold back one of their CTAs.
 * Set it before the stage runs; 0 by default. */
int mg_reserve_sms(int32_t device, int32_t n);

/* Queue a copy of `bytes` from `src` on `src_device` to `dst` on `dst_device`
 * on `stream`, a stream of `src_device` (cudaMemcpyPeerAsync, issued with
 * `src_device` current: direct over NVLink when peer access is enabled). */
int mg_peer_copy(void* dst, int32_t dst_device, const void* src, int32_t src_device, uint64_t bytes,
                 void* stream);

/* ---- Sampling (inference/sampling.py) ---- */

/* Greedy: ids[r] = argmax over logits row r, lowest index on ties
 * (greedy_sample, sampling.py:58-60).  logits [rows, vocab] in `dtype`
 * with row stride `row_stride` elements. */
int mg_sample_greedy(const void* logits, int32_t dtype, int32_t rows, int32_t vocab,
                     int64_t row_stride, int64_t* ids, void* stream);

/* Top-p with temperature (top_p_sample, sampling.py:63-95): probabilities of
 * logits/temperature in fp32, the smallest descending-probability prefix whose
 * exclusive cumulative mass is <= top_p, renormalised, then the token where the
 * cumulative mass of that prefix first reaches uniforms[r] (fp32, [rows], in
 * [0,1)).  Ties in probability are ordered by token index.  temperature <= 0
 * falls back to greedy as the reference does. */
int mg_sample_top_p(const void* logits, int32_t dtype, int32_t rows, int32_t vocab,
                    int64_t row_stride, float temperature, float top_p, const float* uniforms,
                    int64_t* ids, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MESHGPU_B200_H */
