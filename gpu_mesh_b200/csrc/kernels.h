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

// The KV tensor maps of a slot view its block as a 2-D bf16 array
// [layers*2*rows*nkv*cap, D] with a 128-byte swizzle: at kv_tmap a box of
// kKvBoxKeys keys x 64 dims, at kv_tmap + sizeof(CUtensorMap) a box of
// kKvTailKeys keys (the last, partly visible chunk of a sequence is loaded in
// such slices, in the same shared-memory layout); kv_row() is the row of
// (layer, K|V, row, head, pos).
constexpr int kKvBoxKeys = 128;
constexpr int kKvTailKeys = 16;
__host__ __device__ inline int64_t kv_row(int layer, int kv, int slot_rows, int row, int nkv,
                                          int head, int cap, int pos) {
  return ((((int64_t)(layer * 2 + kv) * slot_rows + row) * nkv + head) * cap + pos);
}

// KV block layout of a slot: [local_layer][2 (K,V)][slot_rows][nkv][cap][D].
__host__ __device__ inline size_t kv_offset_elems(int layer, int kv, int slot_rows, int row,
                                                  int nkv, int head, int cap, int D, int pos) {
  return ((((size_t)(layer * 2 + kv) * slot_rows + row) * nkv + head) * cap + pos) * D;
}

// Threads of a row in the RMSNorm kernels; their reduction order is part of
// the result (see block_sum in k_elementwise.cu).
constexpr int kNormThreads = 512;

// Linear epilogues: Y = f(X · Wᵀ).
enum Epilogue : int {
  kEpiStore = 0,   // Y = round(acc)
  kEpiResid = 1,   // Y = round(R + round(acc))            (o_proj / down_proj + residual)
  kEpiSwiGLU = 2,  // Y[:, n] = round(round(silu(round(acc_gate))) * round(acc_up))
  kEpiPieces = 3,  // decode GEMM only: every CTA's fp32 sums left as pieces (see Pieces)
  kEpiGreedy = 4,  // decode GEMM only (lm_head): kEpiStore (Y may be NULL) + per-row argmax (see Greedy)
  kEpiHist = 5,    // decode GEMM only (lm_head): kEpiStore + per-row histogram of the bf16 logits (top-p)
};

// Greedy selection fused into the lm_head decode GEMM.  Every CTA folds the
// rounded logits of the tiles it finishes into best[m], one 64-bit atomic max
// per token row and warp of a packed key (order-preserving bits of the bf16
// logit << 32 | ~vocab index: the largest logit, then the lowest index, as
// torch.argmax); the last CTA to finish (counted in *done) writes
// ids[m] = the index, and returns best[] and *done to zero.
struct Greedy {
  unsigned long long* best;  // [32], zero between launches
  int* done;                 // zero between launches
  int64_t* ids;              // [M] token ids out
};

// The fp32 pieces a decode GEMM leaves with kEpiPieces: the stream-K split
// of tiles x K blocks over G CTAs (tile t = W rows 128t .. 128t + 127), and
// CTA c's sums for tile t at slots[((c + t) · np + m) · 128 + r] for token m,
// row r.  The kernel that consumes the output adds the pieces of a tile in
// CTA order, which is the order the GEMM's own fix-up uses, so the results
// are the same bits.
struct Pieces {
  const float* slots;
  long long total;  // tiles · nk units
  int G, nk, np;
};

__host__ __device__ inline void pieces_range(const Pieces& p, int t, int& c_lo, int& c_hi) {
  c_lo = (int)((((long long)t * p.nk + 1) * p.G - 1) / p.total);
  c_hi = (int)((((long long)(t + 1) * p.nk) * p.G - 1) / p.total);
}

#ifdef __CUDACC__
// Sum of the pieces for token m, W rows f .. f + 7 (f a multiple of 8).
__device__ inline void pieces_sum8(const Pieces& p, int m, int f, float* out) {
  const int t = f >> 7, r = f & 127;
  int c_lo, c_hi;
  pieces_range(p, t, c_lo, c_hi);
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = 0.f;
  for (int c0 = c_lo; c0 <= c_hi; c0 += 8) {
    float4 buf[8][2];  // eight pieces' loads in flight, added in order below
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (c0 + k > c_hi) break;
      const float4* s = reinterpret_cast<const float4*>(p.slots + ((size_t)(c0 + k + t) * p.np + m) * 128 + r);
      buf[k][0] = __ldcg(s);
      buf[k][1] = __ldcg(s + 1);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (c0 + k > c_hi) break;
      out[0] += buf[k][0].x; out[1] += buf[k][0].y; out[2] += buf[k][0].z; out[3] += buf[k][0].w;
      out[4] += buf[k][1].x; out[5] += buf[k][1].y; out[6] += buf[k][1].z; out[7] += buf[k][1].w;
    }
  }
}

// Sum of the pieces for token m, W rows f .. f + 3 (f a multiple of 4).
__device__ inline void pieces_sum4(const Pieces& p, int m, int f, float* out) {
  const int t = f >> 7, r = f & 127;
  int c_lo, c_hi;
  pieces_range(p, t, c_lo, c_hi);
#pragma unroll
  for (int i = 0; i < 4; ++i) out[i] = 0.f;
  for (int c0 = c_lo; c0 <= c_hi; c0 += 8) {
    float4 buf[8];  // eight pieces' loads in flight, added in order below
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (c0 + k > c_hi) break;
      buf[k] = __ldcg(reinterpret_cast<const float4*>(p.slots + ((size_t)(c0 + k + t) * p.np + m) * 128 + r));
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (c0 + k > c_hi) break;
      out[0] += buf[k].x; out[1] += buf[k].y; out[2] += buf[k].z; out[3] += buf[k].w;
    }
  }
}
#endif

// The split a kEpiPieces decode GEMM of this shape uses (slots not set);
// false if the shape does not run on the decode GEMM.
bool gemv_pieces_plan(int dtype, int M, int N, int K, Pieces* out);

// x[m] = round(x[m] + round(pieces[m])) for the M rows of a residual stream
// [M, H] (the o_proj / down_proj residual epilogue), then, if w is not NULL,
// xn[m] = RMSNorm(x[m]) · w with the reduction order of the RMSNorm kernel.
cudaError_t launch_resid_norm_pieces(int dtype, const Pieces& pc, void* x, const void* w, void* xn, int M,
                                     int H, float eps, cudaStream_t s);

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
  // kEpiGreedy: the selection buffers (device pointers; unused otherwise).
  Greedy greedy{nullptr, nullptr, nullptr};
  // kEpiHist: [M][kHistBins] counts of each row's logits by bf16 value, zero
  // when the launch starts (launch_top_p_select clears what it reads).
  int* hist = nullptr;
};

// Top-p over bf16 logits by value histogram: a bf16 logit has one of 65536
// bit patterns, and every token of one value has the same probability, so a
// row's histogram of values holds its whole sorted distribution.
constexpr int kHistBins = 65536;

// A zeroed [rows][kHistBins] int buffer of the current device, grown on
// demand (growth synchronises the device once); NULL on allocation failure.
int* top_p_hist_buffer(int rows);

// Count each bf16 logit of `rows` rows into hist (the histogram half of
// launch_top_p, for logits that were not counted by the lm_head epilogue).
cudaError_t launch_logit_hist(const void* logits, int rows, int vocab, int64_t row_stride, int* hist,
                              cudaStream_t s);

// From each row's histogram and bf16 logits: the top-p token for uniform
// uniforms[r] (the rule of launch_top_p), into ids; clears the histograms.
cudaError_t launch_top_p_select(const void* logits, int rows, int vocab, int64_t row_stride, int* hist,
                                float temperature, float top_p, const float* uniforms, int64_t* ids,
                                cudaStream_t s);

// Scratch (fp32 elements) that launch_linear needs for the given shape.
size_t linear_scratch_elems(int dtype, int M, int N, int K, int epilogue);
cudaError_t launch_linear(const LinearArgs& a, cudaStream_t s);

// Bounded wait on `flag` for `limit_ns`; code 3 in `err` on expiry.
cudaError_t launch_wait_probe(const int* flag, uint64_t limit_ns, int* err, cudaStream_t s);

cudaError_t launch_embed(int dtype, const void* table, const int64_t* ids, int M, int H, int V,
                         void* out, int* err, cudaStream_t s);

// y[m] = RMSNorm(x[m * x_row_stride]) for m < M.
cudaError_t launch_rmsnorm(int dtype, const void* x, int64_t x_row_stride, const void* w, int M,
                           int H, float eps, void* y, cudaStream_t s);

struct QkvPostArgs {
  int dtype;
  const void* qkv;         // [M, (nq + 2 nkv) * D]
  int use_pieces;          // read the qkv projection as pieces (bf16 decode) instead of `qkv`
  Pieces pieces;
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
// Prefill / multi-token attention with query tiles on tcgen05
// (k_attention_prefill_tc.cu): bf16, head_dim 64 or 128, G dividing 16,
// S >= 8 query tokens per row; scores and output in TMEM.
bool attention_prefill_tc_applicable(int dtype, int D, int G, int S);
cudaError_t launch_attention_prefill_tc(const AttnArgs& a, cudaStream_t s);
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
