// Host-side launchers of the stage kernels (internal to the library).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mg {

// Count `n` kernel launches (process-wide, read by mg_launch_count).
void note_launch(int n = 1);

// Launch `kernel` with programmatic stream serialisation (see pdl_wait /
// pdl_trigger in common.cuh) and count it.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  note_launch();
  return e;
}

// One sequence row of a forward batch: where its KV cache lives and how long
// it was before this forward.  Kept in device memory so that a captured decode
// step reads the current lengths instead of baking them in.
struct RowDesc {
  uint64_t kv_base;   // device address of the slot's KV block
  uint64_t kv_tmap;   // device address of the slot's KV tensor map (bf16 D 64/128), or 0
  int32_t slot_rows;  // rows (batch) of the slot
  int32_t row;        // this row's index inside the slot
  int32_t cap;        // positions the slot can hold
  int32_t past;       // cached positions before this forward
};

// The KV tensor map of a slot views its block as a 2-D bf16 array
// [layers*2*rows*nkv*cap, D] with a box of kKvBoxKeys keys x 64 dims and a
// 128-byte swizzle; kv_row() is the row of (layer, K|V, row, head, pos).
constexpr int kKvBoxKeys = 128;
__host__ __device__ inline int64_t kv_row(int layer, int kv, int slot_rows, int row, int nkv,
                                          int head, int cap, int pos) {
  return ((((int64_t)(layer * 2 + kv) * slot_rows + row) * nkv + head) * cap + pos);
}

// KV block layout of a slot: [local_layer][2 (K,V)][slot_rows][nkv][cap][D].
__host__ __device__ inline size_t kv_offset_elems(int layer, int kv, int slot_rows, int row,
                                                  int nkv, int head, int cap, int D, int pos) {
  return ((((size_t)(layer * 2 + kv) * slot_rows + row) * nkv + head) * cap + pos) * D;
}

// Linear epilogues: Y = f(X · Wᵀ).
enum Epilogue : int {
  kEpiStore = 0,   // Y = round(acc)
  kEpiResid = 1,   // Y = round(R + round(acc))            (o_proj / down_proj + residual)
  kEpiSwiGLU = 2,  // Y[:, n] = round(round(silu(round(acc_gate))) * round(acc_up))
};

// Attention mask policies.
enum MaskPolicy : int {
  kMaskSdpa = 0,         // Llama sdpa: single-token query sees every key; else key j <= position
  kMaskEager = 1,        // Llama eager: key j <= position
  kMaskCacheCausal = 2,  // HF causal mask: key j <= past + s
};

struct LinearArgs {
  int dtype;
  const void* X; int64_t ldx;   // [M, K], row stride ldx elements
  const void* W;                // [N, K] (kEpiSwiGLU: [2*N, K], gate rows then up rows)
  void* Y; int64_t ldy;         // [M, N]
  const void* R; int64_t ldr;   // residual for kEpiResid (may alias Y)
  int M, N, K;
  int epilogue;
  float* partial;               // split-K scratch, fp32
  size_t partial_elems;         // capacity of `partial`
  int* err;                     // stage error word (bounded-wait timeouts)
  // Tile counters of the stream-K decode GEMM.  They must be zero when a
  // launch starts and are zero again when it ends.  NULL: carved from the
  // front of `partial` and cleared by the launcher before every launch.
  int* counters;
  size_t counters_elems;
};

// Scratch (fp32 elements) that launch_linear needs for the given shape.
size_t linear_scratch_elems(int dtype, int M, int N, int K, int epilogue);
cudaError_t launch_linear(const LinearArgs& a, cudaStream_t s);

cudaError_t launch_embed(int dtype, const void* table, const int64_t* ids, int M, int H, int V,
                         void* out, int* err, cudaStream_t s);

// y[m] = RMSNorm(x[m * x_row_stride]) for m < M.
cudaError_t launch_rmsnorm(int dtype, const void* x, int64_t x_row_stride, const void* w, int M,
                           int H, float eps, void* y, cudaStream_t s);

struct QkvPostArgs {
  int dtype;
  const void* qkv;         // [M, (nq + 2 nkv) * D]
  const int64_t* positions;// [M] or NULL (position = past + s)
  const RowDesc* rows;     // [B]
  const void* q_norm;      // [D] or NULL
  const void* k_norm;      // [D] or NULL
  const void* cos;         // [max_pos, D/2]
  const void* sin;
  void* q_out;             // [M, nq, D]
  int* err;
  int B, S, nq, nkv, D, layer, max_pos;
  float eps;
};
cudaError_t launch_qkv_post(const QkvPostArgs& a, cudaStream_t s);

struct AttnArgs {
  int dtype;
  const void* q;            // [M, nq, D]
  const int64_t* positions; // [M] or NULL
  const RowDesc* rows;      // [B]
  void* out;                // [M, nq, D]
  float* partial;           // split scratch
  size_t partial_elems;
  int B, S, nq, nkv, D, layer, mask;
  int max_keys;             // upper bound of keys any row can see (past + S)
  float scale;
  int* err;                 // stage error word (bounded-wait timeouts)
  int use_tc;               // every row has a KV tensor map: tensor-core kernel
  // Per-(token, KV head) counters of the tensor-core kernel: zero when a
  // launch starts and zero again when it ends.
  int* counters;
  size_t counters_elems;
};
size_t attention_scratch_elems(int M, int nq, int D, int max_keys);
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s);

// Tensor-core attention (k_attention_tc.cu): bf16, head_dim 64 or 128, G <= 8;
// `splits` 128-key chunks per (token, KV head) of the longest row.  It writes
// `out` itself (no combine launch); its fp32 scratch need is
// attention_tc_scratch_elems, its counters one per (token, KV head).
bool attention_tc_applicable(int dtype, int D, int G);
size_t attention_tc_scratch_elems(int nq, int D);
cudaError_t launch_attention_tc(const AttnArgs& a, int splits, cudaStream_t s);

cudaError_t launch_argmax(int dtype, const void* logits, int rows, int vocab, int64_t row_stride,
                          int64_t* ids, cudaStream_t s);
cudaError_t launch_top_p(int dtype, const void* logits, int rows, int vocab, int64_t row_stride,
                         float temperature, float top_p, const float* uniforms, int64_t* ids,
                         cudaStream_t s);

// Copy [slot_rows, nkv, len, D] K or V of one layer in or out of a slot.
cudaError_t launch_kv_copy(int dtype, void* kv_base, int layer, int kv, int slot_rows, int nkv,
                           int cap, int D, int len, void* ext, bool to_slot, cudaStream_t s);

}  // namespace mg
