// C-ABI stage runtime: weights, KV slots, work buffers and the layer loop.
//
// The layer loop mirrors LlamaDecoderLayer.forward (models/llama_dense.py:259-281)
// and LlamaStage.forward (:350-578):
//   x = embed(ids) | hidden
//   per layer: xn = RMSNorm(x); q,k,v = proj(xn); RoPE; cache append;
//              a = attention(q, K, V); x = x + o_proj(a);
//              xn = RMSNorm(x); x = x + down(silu(gate(xn)) * up(xn))
//   last stage: logits = lm_head(RMSNorm(x))
// with q/k/v fused into one [nq*D + 2*nkv*D, H] weight and gate/up into one
// [2*I, H] weight, packed once when the stage is created.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "linear_tc.h"
#include "tc_common.cuh"
#include "meshgpu_b200.h"

using namespace mg;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MG_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define MG_CUDA(call, what)                       \
  do {                                            \
    cudaError_t _e = (call);                      \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

}  // namespace

namespace mg {

std::atomic<int> g_reserved_sms[64];

int usable_sms() {
  static int full[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!full[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    full[dev] = v > 0 ? v : 148;
  }
  const int n = full[dev] - g_reserved_sms[dev].load();
  return n > 1 ? n : 1;
}

}  // namespace mg

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct LayerW {
  void *ln1, *wqkv, *qn, *kn, *wo, *ln2, *wgu, *wd;
};

struct Slot {
  int batch = 0, cap = 0, len = 0;
  void* kv = nullptr;
  size_t bytes = 0;
  void* tmap = nullptr;  // device copies of the two KV tensor maps (bf16, D 64/128), or NULL
};

struct ProfRec {
  int cls;
  cudaEvent_t a, b;
  double bytes, flops;
};

std::atomic<uint64_t> g_launches{0};

// Pinned staging ring for the per-forward row table, so uploading it never
// waits for the device.
struct RowRing {
  static constexpr int kEntries = 8;
  RowDesc* host = nullptr;
  cudaEvent_t ev[kEntries] = {};
  int cap_rows = 0, next = 0;
};

}  // namespace

struct mg_stage {
  mg_stage_config cfg{};
  int L = 0, nq = 0, nkv = 0, D = 0, H = 0, I = 0, V = 0, Nqkv = 0;
  size_t esz = 0;
  void* wbuf = nullptr;
  size_t wbytes = 0;
  void *embed = nullptr, *norm = nullptr, *lm_head = nullptr, *cos = nullptr, *sin = nullptr;
  std::vector<LayerW> layers;
  std::map<int, Slot> slots;
  size_t kv_bytes = 0;
  // Work buffers.
  void* work = nullptr;
  size_t work_bytes = 0;
  int work_tokens = 0, work_rows = 0;
  size_t work_scratch = 0;
  int* counters = nullptr;  // stream-K tile counters: zero between launches
  size_t counters_elems = 0;
  // Greedy selection fused into lm_head (Greedy): zero between launches.
  unsigned long long* greedy_best = nullptr;
  int* greedy_done = nullptr;
  // Logits of a greedy decode whose caller wants only token ids, when the
  // selection cannot be fused (kept between calls, grown on demand).
  void* greedy_logits = nullptr;
  size_t greedy_logits_bytes = 0;
  void *x = nullptr, *xn = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr, *h = nullptr;
  float* part = nullptr;
  RowDesc* rows = nullptr;
  int* err = nullptr;
  RowRing ring;
  // Instrumentation (mg_stage_profile).
  bool profiling = false;
  std::vector<ProfRec> prof_pending;
  std::vector<cudaEvent_t> ev_pool;
  mg_profile prof{};
};

namespace mg {
void note_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }
}  // namespace mg

namespace {

int validate_config(const mg_stage_config& c) {
  const int32_t pos[] = {c.vocab_size, c.hidden_size, c.intermediate_size, c.num_hidden_layers,
                         c.num_attention_heads, c.num_key_value_heads, c.head_dim,
                         c.max_position_embeddings};
  const char* names[] = {"vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
                         "num_attention_heads", "num_key_value_heads", "head_dim",
                         "max_position_embeddings"};
  for (int i = 0; i < 8; ++i)
    if (pos[i] < 1) return fail(MG_EINVAL, "%s must be positive, got %d", names[i], pos[i]);
  if (c.num_attention_heads % c.num_key_value_heads != 0)
    return fail(MG_EINVAL,
                "num_attention_heads must be divisible by num_key_value_heads (%d %% %d != 0)",
                c.num_attention_heads, c.num_key_value_heads);
  if (c.head_dim % 2 != 0)
    return fail(MG_EINVAL, "head_dim must be even for rotary embeddings, got %d", c.head_dim);
  if (!(c.rms_norm_eps > 0.f)) return fail(MG_EINVAL, "rms_norm_eps must be positive");
  if (c.dtype != MG_DTYPE_F32 && c.dtype != MG_DTYPE_BF16)
    return fail(MG_EINVAL, "dtype must be MG_DTYPE_F32 or MG_DTYPE_BF16");
  if (c.attention_impl < 0 || c.attention_impl > 2)
    return fail(MG_EINVAL, "attention_impl must be 0 (sdpa), 1 (eager) or 2 (cache-causal)");
  if (!(0 <= c.layer_start && c.layer_start < c.layer_end && c.layer_end <= c.num_hidden_layers))
    return fail(MG_EINVAL, "invalid layer range [%d, %d) for %d layers", c.layer_start,
                c.layer_end, c.num_hidden_layers);
  // Geometry the kernels are built for.
  const int D = c.head_dim;
  if (!(D == 8 || D == 16 || D == 32 || D == 64 || D == 128) || (c.dtype == MG_DTYPE_F32 && D < 8))
    return fail(MG_EINVAL, "head_dim must be one of 8, 16, 32, 64, 128 (got %d)", D);
  if (c.num_attention_heads / c.num_key_value_heads > 8)
    return fail(MG_EINVAL, "at most 8 query heads per KV head are supported (got %d)",
                c.num_attention_heads / c.num_key_value_heads);
  if (c.hidden_size % 8 != 0 || c.intermediate_size % 8 != 0)
    return fail(MG_EINVAL, "hidden_size and intermediate_size must be multiples of 8");
  return MG_OK;
}

int ensure_ring(mg_stage* st, int rows) {
  RowRing& r = st->ring;
  if (rows <= r.cap_rows) return MG_OK;
  if (r.host) {
    for (int i = 0; i < RowRing::kEntries; ++i) cudaEventSynchronize(r.ev[i]);
    cudaFreeHost(r.host);
    r.host = nullptr;
  }
  const int cap = std::max(rows, 64);
  MG_CUDA(cudaMallocHost((void**)&r.host, sizeof(RowDesc) * cap * RowRing::kEntries),
          "cudaMallocHost(row ring)");
  for (int i = 0; i < RowRing::kEntries; ++i)
    if (!r.ev[i]) MG_CUDA(cudaEventCreateWithFlags(&r.ev[i], cudaEventDisableTiming), "event");
  r.cap_rows = cap;
  return MG_OK;
}

size_t scratch_needed(const mg_stage* st, int M, int rows, int max_keys) {
  const int dt = st->cfg.dtype;
  size_t s = 0;
  s = std::max(s, linear_scratch_elems(dt, M, st->Nqkv, st->H, kEpiStore));
  s = std::max(s, linear_scratch_elems(dt, M, st->H, st->nq * st->D, kEpiResid));
  s = std::max(s, linear_scratch_elems(dt, M, st->I, st->H, kEpiSwiGLU));
  s = std::max(s, linear_scratch_elems(dt, M, st->H, st->I, kEpiResid));
  if (st->cfg.has_lm_head) {
    s = std::max(s, linear_scratch_elems(dt, M, st->V, st->H, kEpiStore));
    s = std::max(s, linear_scratch_elems(dt, rows, st->V, st->H, kEpiStore));
  }
  s = std::max(s, attention_scratch_elems(M, st->nq, st->D, max_keys));
  if (M <= 32) {
    s = std::max(s, linear_scratch_elems(dt, M, st->Nqkv, st->H, kEpiPieces));
    s = std::max(s, linear_scratch_elems(dt, M, st->H, st->nq * st->D, kEpiPieces));
    s = std::max(s, linear_scratch_elems(dt, M, st->H, st->I, kEpiPieces));
  }
  return s;
}

int ensure_work(mg_stage* st, int M, int rows, int max_keys) {
  const size_t need_scratch = scratch_needed(st, M, rows, max_keys);
  if (M <= st->work_tokens && rows <= st->work_rows && need_scratch <= st->work_scratch)
    return MG_OK;
  const int Mt = std::max(M, st->work_tokens);
  const int Rt = std::max(std::max(rows, st->work_rows), 64);
  const size_t scr = std::max(need_scratch, st->work_scratch);
  const size_t e = st->esz;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  const size_t o_x = take((size_t)Mt * st->H * e);
  const size_t o_xn = take((size_t)Mt * st->H * e);
  const size_t o_qkv = take((size_t)Mt * st->Nqkv * e);
  const size_t o_q = take((size_t)Mt * st->nq * st->D * e);
  const size_t o_attn = take((size_t)Mt * st->nq * st->D * e);
  const size_t o_h = take((size_t)Mt * st->I * e);
  const size_t o_part = take(std::max<size_t>(scr, 1) * sizeof(float));
  const size_t o_rows = take((size_t)Rt * sizeof(RowDesc));
  size_t n_counters = 0;
  n_counters = std::max(n_counters, gemv_tc_tiles(st->Nqkv, kEpiStore));
  n_counters = std::max(n_counters, gemv_tc_tiles(st->H, kEpiResid));
  n_counters = std::max(n_counters, gemv_tc_tiles(st->I, kEpiSwiGLU));
  if (st->cfg.has_lm_head) n_counters = std::max(n_counters, gemv_tc_tiles(st->V, kEpiStore));
  n_counters = std::max(n_counters, (size_t)Mt * st->nkv);  // attention: one per (token, KV head)
  const size_t o_counters = take(n_counters * sizeof(int));
  const size_t o_greedy = take(64 * sizeof(unsigned long long));  // best[32], done
  if (st->work) {
    MG_CUDA(cudaDeviceSynchronize(), "synchronize before work resize");
    cudaFree(st->work);
    st->work = nullptr;
  }
  cudaError_t ce = cudaMalloc(&st->work, off);
  if (ce != cudaSuccess) {
    st->work_tokens = st->work_rows = 0;
    st->work_scratch = 0;
    st->work_bytes = 0;
    return fail(MG_ENOMEM, "cannot allocate %zu bytes of work memory: %s", off,
                cudaGetErrorString(ce));
  }
  char* base = (char*)st->work;
  st->x = base + o_x;
  st->xn = base + o_xn;
  st->qkv = base + o_qkv;
  st->q = base + o_q;
  st->attn = base + o_attn;
  st->h = base + o_h;
  st->part = (float*)(base + o_part);
  st->rows = (RowDesc*)(base + o_rows);
  st->counters = (int*)(base + o_counters);
  st->counters_elems = n_counters;
  MG_CUDA(cudaMemset(st->counters, 0, n_counters * sizeof(int)), "zero tile counters");
  st->greedy_best = (unsigned long long*)(base + o_greedy);
  st->greedy_done = (int*)(st->greedy_best + 32);
  MG_CUDA(cudaMemset(st->greedy_best, 0, 64 * sizeof(unsigned long long)), "zero greedy selection");
  st->work_bytes = off;
  st->work_tokens = Mt;
  st->work_rows = Rt;
  st->work_scratch = scr;
  return ensure_ring(st, Rt);
}

size_t slot_bytes(const mg_stage* st, int batch, int cap) {
  return (size_t)st->L * 2 * batch * st->nkv * cap * st->D * st->esz;
}

// Make `slot` hold `batch` rows with room for `need` positions, keeping its
// contents.  A fresh slot gets exactly what is asked; growth doubles.
int reserve_slot(mg_stage* st, int id, int batch, int need, cudaStream_t s) {
  Slot& sl = st->slots[id];
  if (sl.batch == 0) sl.batch = batch;
  if (need <= sl.cap) return MG_OK;
  const int maxp = st->cfg.max_position_embeddings;
  int cap = std::max(need, sl.cap ? 2 * sl.cap : need);
  cap = (int)std::min<size_t>(align_up(cap, 64), (size_t)maxp);
  if (cap < need) cap = need;
  void* kv = nullptr;
  const size_t bytes = slot_bytes(st, sl.batch, cap);
  cudaError_t ce = cudaMalloc(&kv, bytes);
  if (ce != cudaSuccess)
    return fail(MG_ENOMEM, "cannot allocate %zu bytes of KV cache: %s", bytes,
                cudaGetErrorString(ce));
  if (sl.kv && sl.len > 0) {
    const size_t run = (size_t)sl.len * st->D * st->esz;
    const size_t runs = (size_t)st->L * 2 * sl.batch * st->nkv;
    ce = cudaMemcpy2DAsync(kv, (size_t)cap * st->D * st->esz, sl.kv,
                           (size_t)sl.cap * st->D * st->esz, run, runs, cudaMemcpyDeviceToDevice, s);
    if (ce != cudaSuccess) {
      cudaFree(kv);
      return cuda_fail(ce, "KV cache growth copy");
    }
  }
  if (sl.kv) {
    cudaStreamSynchronize(s);
    cudaFree(sl.kv);
    st->kv_bytes -= sl.bytes;
  }
  sl.kv = kv;
  sl.cap = cap;
  sl.bytes = bytes;
  st->kv_bytes += bytes;
  // Tensor maps of the block for the tensor-core attention: a 2-D bf16 view
  // [layers*2*rows*nkv*cap, D], one with a box of kKvBoxKeys keys x 64 dims
  // and, right after it, one with a box of kKvTailKeys keys for the partly
  // visible last chunk of a sequence.
  if (attention_tc_applicable(st->cfg.dtype, st->D, st->nq / st->nkv)) {
    CUtensorMap tm[2];
    const uint64_t rows = (uint64_t)st->L * 2 * sl.batch * st->nkv * cap;
    if (rows < (1ull << 31) && tc_host::make_map(&tm[0], kv, rows, st->D, st->D, kKvBoxKeys) &&
        tc_host::make_map(&tm[1], kv, rows, st->D, st->D, kKvTailKeys)) {
      if (!sl.tmap) MG_CUDA(cudaMalloc(&sl.tmap, sizeof(tm)), "KV tensor map");
      MG_CUDA(cudaMemcpy(sl.tmap, tm, sizeof(tm), cudaMemcpyHostToDevice), "KV tensor map upload");
    } else if (sl.tmap) {
      cudaFree(sl.tmap);
      sl.tmap = nullptr;
    }
  }
  return MG_OK;
}

void drop_slot(mg_stage* st, int id) {
  auto it = st->slots.find(id);
  if (it == st->slots.end()) return;
  if (it->second.kv) {
    cudaDeviceSynchronize();
    cudaFree(it->second.kv);
    st->kv_bytes -= it->second.bytes;
  }
  if (it->second.tmap) cudaFree(it->second.tmap);
  st->slots.erase(it);
}

// Upload the row table through the pinned ring.
int upload_rows(mg_stage* st, const std::vector<RowDesc>& rows, cudaStream_t s) {
  RowRing& r = st->ring;
  const int e = r.next;
  r.next = (r.next + 1) % RowRing::kEntries;
  MG_CUDA(cudaEventSynchronize(r.ev[e]), "row ring wait");
  RowDesc* h = r.host + (size_t)e * r.cap_rows;
  std::memcpy(h, rows.data(), rows.size() * sizeof(RowDesc));
  MG_CUDA(cudaMemcpyAsync(st->rows, h, rows.size() * sizeof(RowDesc), cudaMemcpyHostToDevice, s),
          "row table upload");
  MG_CUDA(cudaEventRecord(r.ev[e], s), "row ring record");
  return MG_OK;
}

#define MG_LAUNCH(call, what)                          \
  do {                                                 \
    cudaError_t _e = (call);                           \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

cudaEvent_t prof_event(mg_stage* st) {
  if (!st->ev_pool.empty()) {
    cudaEvent_t e = st->ev_pool.back();
    st->ev_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

int prof_collect(mg_stage* st) {
  for (ProfRec& r : st->prof_pending) {
    MG_CUDA(cudaEventSynchronize(r.b), "profile event wait");
    float ms = 0.f;
    MG_CUDA(cudaEventElapsedTime(&ms, r.a, r.b), "profile event time");
    st->prof.ms[r.cls] += ms;
    st->prof.bytes[r.cls] += r.bytes;
    st->prof.flops[r.cls] += r.flops;
    st->prof.launches[r.cls] += 1;
    st->ev_pool.push_back(r.a);
    st->ev_pool.push_back(r.b);
  }
  st->prof_pending.clear();
  return MG_OK;
}

// Launch `call`; while profiling, bracket it with events and book its
// algorithmic bytes / FLOPs under class `cls`.
#define MG_TIMED(cls, nbytes, nflops, call, what)                                    \
  do {                                                                                 \
    cudaEvent_t _a = nullptr;                                                          \
    if (st->profiling) {                                                               \
      _a = prof_event(st);                                                             \
      cudaEventRecord(_a, s);                                                          \
    }                                                                                  \
    MG_LAUNCH(call, what);                                                             \
    if (st->profiling) {                                                               \
      cudaEvent_t _b = prof_event(st);                                                 \
      cudaEventRecord(_b, s);                                                          \
      st->prof_pending.push_back(ProfRec{cls, _a, _b, (double)(nbytes), (double)(nflops)}); \
    }                                                                                  \
  } while (0)

double linear_bytes(const LinearArgs& a, size_t esz) {
  const double wrows = a.epilogue == kEpiSwiGLU ? 2.0 * a.N : (double)a.N;
  const double out = (double)a.M * a.N * (a.epilogue == kEpiResid ? 2 : 1);
  return (wrows * a.K + (double)a.M * a.K + out) * esz;
}
double linear_flops(const LinearArgs& a) {
  const double wrows = a.epilogue == kEpiSwiGLU ? 2.0 * a.N : (double)a.N;
  return 2.0 * a.M * wrows * a.K;
}
int linear_class(const LinearArgs& a) {
  return a.M <= 32 ? MG_PROF_LINEAR_DECODE : MG_PROF_LINEAR_PREFILL;
}

// The layer loop for one batch of rows sharing the query length S.
// `greedy_ids` (device int64 [rows of logits], last stage only): also select
// each row's greedy token, fused into lm_head where the decode GEMM runs it;
// `out` may then be NULL when the logits themselves are not wanted.
struct TopPSel {
  float temperature, top_p;
  const float* uniforms;  // [rows] in [0, 1)
  int64_t* ids;           // [rows] out
};

int run_stage(mg_stage* st, const std::vector<RowDesc>& rows, int S, const int64_t* ids,
              const void* hidden_in, const int64_t* positions, int out_mode, void* out,
              cudaStream_t s, int64_t* greedy_ids = nullptr, const TopPSel* tp = nullptr) {
  const mg_stage_config& c = st->cfg;
  const int B = (int)rows.size();
  const int M = B * S;
  int max_keys = 0;
  for (const RowDesc& r : rows) max_keys = std::max(max_keys, r.past + S);
  int rc = ensure_work(st, M, B, max_keys);
  if (rc) return rc;
  rc = upload_rows(st, rows, s);
  if (rc) return rc;

  const int dt = c.dtype;
  const int H = st->H;
  if (c.has_embedding) {
    MG_TIMED(MG_PROF_OTHER, 2.0 * M * H * st->esz, 0, launch_embed(dt, st->embed, ids, M, H, st->V, st->x, st->err, s), "embedding");
  } else {
    MG_CUDA(cudaMemcpyAsync(st->x, hidden_in, (size_t)M * H * st->esz, cudaMemcpyDeviceToDevice, s),
            "hidden input copy");
  }

  LinearArgs la{};
  la.dtype = dt;
  la.partial = st->part;
  la.partial_elems = st->work_scratch;
  la.err = st->err;
  la.counters = st->counters;
  la.counters_elems = st->counters_elems;
  la.M = M;

  QkvPostArgs qa{};
  qa.dtype = dt;
  qa.qkv = st->qkv;
  qa.positions = positions;
  qa.rows = st->rows;
  qa.cos = st->cos;
  qa.sin = st->sin;
  qa.q_out = st->q;
  qa.err = st->err;
  qa.B = B;
  qa.S = S;
  qa.nq = st->nq;
  qa.nkv = st->nkv;
  qa.D = st->D;
  qa.max_pos = c.max_position_embeddings;
  qa.eps = c.rms_norm_eps;

  AttnArgs aa{};
  aa.dtype = dt;
  aa.q = st->q;
  aa.positions = positions;
  aa.rows = st->rows;
  aa.out = st->attn;
  aa.partial = st->part;
  aa.partial_elems = st->work_scratch;
  aa.B = B;
  aa.S = S;
  aa.nq = st->nq;
  aa.nkv = st->nkv;
  aa.D = st->D;
  aa.mask = c.attention_impl;
  aa.max_keys = max_keys;
  aa.scale = 1.0f / sqrtf((float)st->D);
  aa.err = st->err;
  aa.use_tc = 1;
  for (const RowDesc& r : rows) aa.use_tc &= r.kv_tmap != 0;
  aa.counters = st->counters;
  aa.counters_elems = st->counters_elems;

  const int qd = st->nq * st->D;
  const double norm_bytes = 2.0 * M * H * st->esz;
  double attn_bytes = 2.0 * M * qd * st->esz, attn_flops = 0.0;
  for (const RowDesc& r : rows) {
    attn_bytes += 2.0 * st->nkv * (double)(r.past + S) * st->D * st->esz;
    for (int q = 0; q < S; ++q) {
      const double vis = (S == 1) ? (double)(r.past + 1) : (double)(r.past + q + 1);
      attn_flops += 4.0 * vis * qd;
    }
  }
  const bool last_only = out_mode == MG_OUT_LOGITS_LAST;
  const int rows_out = last_only ? B : M;
  const bool fuse_greedy = greedy_ids && c.has_lm_head && gemv_tc_applicable(dt, rows_out, st->V, H);
  // Top-p rows: the lm_head's epilogue counts the bf16 logits by value
  // (kEpiHist) and one selection kernel draws from the histograms.
  const bool fuse_hist = tp && c.has_lm_head && dt == kBF16 && gemv_tc_applicable(dt, rows_out, st->V, H);
  int* hist = nullptr;
  if (tp && dt == kBF16) {
    hist = top_p_hist_buffer(rows_out);
    if (!hist) return fail(MG_ENOMEM, "top-p histogram buffer");
  }
  if (greedy_ids && c.has_lm_head && !out && !fuse_greedy) {
    // the selection reads the logits: give them somewhere to go
    const size_t need = (size_t)rows_out * st->V * st->esz;
    if (need > st->greedy_logits_bytes) {
      if (st->greedy_logits) {
        MG_CUDA(cudaStreamSynchronize(s), "synchronize before logits buffer resize");
        cudaFree(st->greedy_logits);
        st->greedy_logits = nullptr;
        st->greedy_logits_bytes = 0;
      }
      MG_CUDA(cudaMalloc(&st->greedy_logits, need), "greedy logits buffer");
      st->greedy_logits_bytes = need;
    }
    out = st->greedy_logits;
  }
  bool final_norm_done = false;  // the last residual kernel also ran the final norm
  {
    // Decode rows on the tcgen05 GEMM: the qkv, o_proj and down projections
    // leave their fp32 pieces, and the kernel after each (RoPE / append, or
    // the residual add + RMSNorm) adds them, so no GEMM ends in a fix-up.
    Pieces pq{}, po{}, pd{};
    const bool use_pieces = M <= 32 && gemv_pieces_plan(dt, M, st->Nqkv, H, &pq) &&
                            gemv_pieces_plan(dt, M, H, qd, &po) && gemv_pieces_plan(dt, M, H, st->I, &pd);
    pq.slots = po.slots = pd.slots = st->part;
    const double resid_bytes = 3.0 * M * H * st->esz;  // residual in and out, normalised row out
    for (int l = 0; l < st->L; ++l) {
      const LayerW& w = st->layers[l];
      if (l == 0 || !use_pieces)
        MG_TIMED(MG_PROF_OTHER, norm_bytes, 0, launch_rmsnorm(dt, st->x, H, w.ln1, M, H, c.rms_norm_eps, st->xn, s), "input_layernorm");
      la.X = st->xn; la.ldx = H; la.W = w.wqkv; la.Y = st->qkv; la.ldy = st->Nqkv;
      la.N = st->Nqkv; la.K = H; la.epilogue = use_pieces ? kEpiPieces : kEpiStore; la.R = nullptr;
      qa.layer = l;
      qa.q_norm = w.qn;
      qa.k_norm = w.kn;
      qa.use_pieces = use_pieces;
      qa.pieces = pq;
      if (qkv_rope_fusable(la, qa)) {  // prefill: RoPE and the KV append in the projection's epilogue
        MG_TIMED(linear_class(la), linear_bytes(la, st->esz), linear_flops(la), launch_qkv_rope_kv(la, qa, s),
                 "qkv projection + rope / kv append");
      } else {
        MG_TIMED(linear_class(la), linear_bytes(la, st->esz), linear_flops(la), launch_linear(la, s), "qkv projection");
        MG_TIMED(MG_PROF_OTHER, 2.0 * M * st->Nqkv * st->esz, 0, launch_qkv_post(qa, s), "rope / kv append");
      }
      aa.layer = l;
      MG_TIMED(MG_PROF_ATTENTION, attn_bytes, attn_flops, launch_attention(aa, s), "attention");
      la.X = st->attn; la.ldx = qd; la.W = w.wo; la.Y = st->x; la.ldy = H;
      la.N = H; la.K = qd; la.epilogue = use_pieces ? kEpiPieces : kEpiResid; la.R = st->x; la.ldr = H;
      MG_TIMED(linear_class(la), linear_bytes(la, st->esz), linear_flops(la), launch_linear(la, s), "o_proj");
      if (use_pieces)
        MG_TIMED(MG_PROF_OTHER, resid_bytes, 0,
                 launch_resid_norm_pieces(dt, po, st->x, w.ln2, st->xn, M, H, c.rms_norm_eps, s),
                 "o_proj residual + post_attention_layernorm");
      else
        MG_TIMED(MG_PROF_OTHER, norm_bytes, 0,
                 launch_rmsnorm(dt, st->x, H, w.ln2, M, H, c.rms_norm_eps, st->xn, s),
                 "post_attention_layernorm");
      la.X = st->xn; la.ldx = H; la.W = w.wgu; la.Y = st->h; la.ldy = st->I;
      la.N = st->I; la.K = H; la.epilogue = kEpiSwiGLU; la.R = nullptr;
      MG_TIMED(linear_class(la), linear_bytes(la, st->esz), linear_flops(la), launch_linear(la, s), "gate/up projection");
      la.X = st->h; la.ldx = st->I; la.W = w.wd; la.Y = st->x; la.ldy = H;
      la.N = H; la.K = st->I; la.epilogue = use_pieces ? kEpiPieces : kEpiResid; la.R = st->x; la.ldr = H;
      MG_TIMED(linear_class(la), linear_bytes(la, st->esz), linear_flops(la), launch_linear(la, s), "down_proj");
      if (use_pieces) {
        const void* nw = nullptr;
        if (l + 1 < st->L) {
          nw = st->layers[l + 1].ln1;
        } else if (c.has_lm_head && rows_out == M) {
          nw = st->norm;
          final_norm_done = true;
        }
        MG_TIMED(MG_PROF_OTHER, resid_bytes, 0,
                 launch_resid_norm_pieces(dt, pd, st->x, nw, st->xn, M, H, c.rms_norm_eps, s),
                 "down_proj residual + next norm");
      }
    }
  }

  if (c.has_lm_head) {
    const void* src = last_only ? (const void*)((const char*)st->x + (size_t)(S - 1) * H * st->esz)
                                : st->x;
    const int64_t stride = last_only ? (int64_t)S * H : H;
    if (!final_norm_done)
      MG_TIMED(MG_PROF_OTHER, 2.0 * rows_out * H * st->esz, 0,
               launch_rmsnorm(dt, src, stride, st->norm, rows_out, H, c.rms_norm_eps, st->xn, s),
               "final norm");
    la.M = rows_out;
    la.X = st->xn; la.ldx = H; la.W = st->lm_head; la.Y = out; la.ldy = st->V;
    la.N = st->V; la.K = H; la.epilogue = fuse_greedy ? kEpiGreedy : fuse_hist ? kEpiHist : kEpiStore;
    la.R = nullptr;
    if (fuse_greedy) la.greedy = Greedy{st->greedy_best, st->greedy_done, greedy_ids};
    if (fuse_hist) la.hist = hist;
    MG_TIMED(linear_class(la), linear_bytes(la, st->esz), linear_flops(la), launch_linear(la, s), "lm_head");
  } else {
    MG_CUDA(cudaMemcpyAsync(out, st->x, (size_t)M * H * st->esz, cudaMemcpyDeviceToDevice, s),
            "hidden output copy");
  }
  if (greedy_ids && c.has_lm_head && !fuse_greedy)
    MG_TIMED(MG_PROF_OTHER, (double)rows_out * st->V * st->esz, 0,
             launch_argmax(dt, out, rows_out, st->V, st->V, greedy_ids, s), "greedy selection");
  if (tp && c.has_lm_head) {
    const double row_bytes = (double)rows_out * st->V * st->esz;
    if (dt != kBF16) {
      MG_TIMED(MG_PROF_OTHER, row_bytes, 0,
               launch_top_p(dt, out, rows_out, st->V, st->V, tp->temperature, tp->top_p, tp->uniforms, tp->ids, s),
               "top-p selection");
    } else {
      if (!fuse_hist)
        MG_TIMED(MG_PROF_OTHER, row_bytes, 0, launch_logit_hist(out, rows_out, st->V, st->V, hist, s),
                 "top-p histogram");
      MG_TIMED(MG_PROF_OTHER, row_bytes + (double)rows_out * kHistBins * 8, 0,
               launch_top_p_select(out, rows_out, st->V, st->V, hist, tp->temperature, tp->top_p,
                                   tp->uniforms, tp->ids, s),
               "top-p selection");
    }
  }
  return MG_OK;
}

int check_out_mode(const mg_stage* st, int out_mode) {
  if (st->cfg.has_lm_head) {
    if (out_mode != MG_OUT_LOGITS_ALL && out_mode != MG_OUT_LOGITS_LAST)
      return fail(MG_EINVAL, "the last stage produces logits (out_mode 1 or 2)");
  } else if (out_mode != MG_OUT_HIDDEN) {
    return fail(MG_EINVAL, "a non-final stage produces hidden states (out_mode 0)");
  }
  return MG_OK;
}

int check_inputs(const mg_stage* st, const int64_t* ids, const void* hidden) {
  if (st->cfg.has_embedding) {
    if (!ids) return fail(MG_EINVAL, "the embedding stage requires input_ids");
  } else {
    if (ids) return fail(MG_EINVAL, "input_ids are only accepted by the embedding stage");
    if (!hidden)
      return fail(MG_EINVAL, "a non-embedding stage requires non-empty hidden states [B, S, H]");
  }
  return MG_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// Exported entry points.
// ---------------------------------------------------------------------------
extern "C" {

const char* mg_version(void) { return "meshgpu_b200 0.1 (sm_100a)"; }

const char* mg_last_error(void) { return g_last_error.c_str(); }

int mg_stage_create(const mg_stage_config* cfg, const mg_stage_weights* w, mg_stage** out) {
  if (!cfg || !w || !out) return fail(MG_EINVAL, "mg_stage_create: null argument");
  *out = nullptr;
  int rc = validate_config(*cfg);
  if (rc) return rc;
  const mg_stage_config& c = *cfg;
  if (!w->rope_cos || !w->rope_sin) return fail(MG_EINVAL, "rope tables are required");
  if (c.has_embedding && !w->embed_tokens) return fail(MG_EINVAL, "embed_tokens is required");
  if (c.has_lm_head && (!w->norm || !w->lm_head))
    return fail(MG_EINVAL, "norm and lm_head are required on the last stage");
  if (!w->layers) return fail(MG_EINVAL, "layer weights are required");

  DeviceGuard guard(c.device);
  mg_stage* st = new mg_stage();
  st->cfg = c;
  st->L = c.layer_end - c.layer_start;
  st->nq = c.num_attention_heads;
  st->nkv = c.num_key_value_heads;
  st->D = c.head_dim;
  st->H = c.hidden_size;
  st->I = c.intermediate_size;
  st->V = c.vocab_size;
  st->Nqkv = (st->nq + 2 * st->nkv) * st->D;
  st->esz = c.dtype == MG_DTYPE_BF16 ? 2 : 4;
  const size_t e = st->esz;
  const size_t H = st->H, I = st->I, D = st->D, V = st->V, qd = (size_t)st->nq * D,
               kd = (size_t)st->nkv * D;

  // Weight arena layout.
  size_t off = 0;
  auto take = [&](size_t elems) {
    const size_t o = off;
    off = align_up(off + elems * e, 256);
    return o;
  };
  const bool tied = c.has_embedding && c.has_lm_head && w->lm_head == w->embed_tokens;
  const size_t o_embed = c.has_embedding ? take(V * H) : 0;
  const size_t o_norm = c.has_lm_head ? take(H) : 0;
  const size_t o_head = (c.has_lm_head && !tied) ? take(V * H) : 0;
  const size_t half = D / 2, maxp = c.max_position_embeddings;
  const size_t o_cos = take(maxp * half);
  const size_t o_sin = take(maxp * half);
  struct LO { size_t ln1, wqkv, qn, kn, wo, ln2, wgu, wd; };
  std::vector<LO> lo(st->L);
  for (int l = 0; l < st->L; ++l) {
    lo[l].ln1 = take(H);
    lo[l].wqkv = take((qd + 2 * kd) * H);
    lo[l].qn = c.qk_norm ? take(D) : 0;
    lo[l].kn = c.qk_norm ? take(D) : 0;
    lo[l].wo = take(H * qd);
    lo[l].ln2 = take(H);
    lo[l].wgu = take(2 * I * H);
    lo[l].wd = take(H * I);
  }
  cudaError_t ce = cudaMalloc(&st->wbuf, off);
  if (ce != cudaSuccess) {
    delete st;
    return fail(MG_ENOMEM, "cannot allocate %zu bytes of stage weights: %s", off,
                cudaGetErrorString(ce));
  }
  st->wbytes = off;
  char* base = (char*)st->wbuf;
  auto cp = [&](size_t dst_off, const void* src, size_t elems) -> cudaError_t {
    return cudaMemcpy(base + dst_off, src, elems * e, cudaMemcpyDefault);
  };
  ce = cudaSuccess;
  auto chain = [&](cudaError_t r) {
    if (ce == cudaSuccess) ce = r;
  };
  if (c.has_embedding) {
    chain(cp(o_embed, w->embed_tokens, V * H));
    st->embed = base + o_embed;
  }
  if (c.has_lm_head) {
    chain(cp(o_norm, w->norm, H));
    st->norm = base + o_norm;
    if (tied) {
      st->lm_head = st->embed;
    } else {
      chain(cp(o_head, w->lm_head, V * H));
      st->lm_head = base + o_head;
    }
  }
  chain(cp(o_cos, w->rope_cos, maxp * half));
  chain(cp(o_sin, w->rope_sin, maxp * half));
  st->cos = base + o_cos;
  st->sin = base + o_sin;
  st->layers.resize(st->L);
  for (int l = 0; l < st->L && ce == cudaSuccess; ++l) {
    const mg_layer_weights& lw = w->layers[l];
    if (!lw.input_layernorm || !lw.q_proj || !lw.k_proj || !lw.v_proj || !lw.o_proj ||
        !lw.post_attention_layernorm || !lw.gate_proj || !lw.up_proj || !lw.down_proj ||
        (c.qk_norm && (!lw.q_norm || !lw.k_norm))) {
      cudaFree(st->wbuf);
      delete st;
      return fail(MG_EINVAL, "layer %d: missing weight pointer", l);
    }
    chain(cp(lo[l].ln1, lw.input_layernorm, H));
    chain(cp(lo[l].wqkv, lw.q_proj, qd * H));
    chain(cp(lo[l].wqkv + qd * H * e, lw.k_proj, kd * H));
    chain(cp(lo[l].wqkv + (qd + kd) * H * e, lw.v_proj, kd * H));
    if (c.qk_norm) {
      chain(cp(lo[l].qn, lw.q_norm, D));
      chain(cp(lo[l].kn, lw.k_norm, D));
    }
    chain(cp(lo[l].wo, lw.o_proj, H * qd));
    chain(cp(lo[l].ln2, lw.post_attention_layernorm, H));
    chain(cp(lo[l].wgu, lw.gate_proj, I * H));
    chain(cp(lo[l].wgu + I * H * e, lw.up_proj, I * H));
    chain(cp(lo[l].wd, lw.down_proj, H * I));
    LayerW& L = st->layers[l];
    L.ln1 = base + lo[l].ln1;
    L.wqkv = base + lo[l].wqkv;
    L.qn = c.qk_norm ? base + lo[l].qn : nullptr;
    L.kn = c.qk_norm ? base + lo[l].kn : nullptr;
    L.wo = base + lo[l].wo;
    L.ln2 = base + lo[l].ln2;
    L.wgu = base + lo[l].wgu;
    L.wd = base + lo[l].wd;
  }
  // err[0]: the error word; err[1]: the probe flag of mg_stage_probe_wait
  if (ce == cudaSuccess) ce = cudaMalloc((void**)&st->err, 2 * sizeof(int));
  if (ce == cudaSuccess) ce = cudaMemset(st->err, 0, 2 * sizeof(int));
  if (ce != cudaSuccess) {
    if (st->err) cudaFree(st->err);
    cudaFree(st->wbuf);
    delete st;
    return cuda_fail(ce, "copying stage weights");
  }
  *out = st;
  return MG_OK;
}

int mg_stage_destroy(mg_stage* st) {
  if (!st) return MG_OK;
  DeviceGuard guard(st->cfg.device);
  cudaDeviceSynchronize();
  for (auto& kv : st->slots) {
    if (kv.second.kv) cudaFree(kv.second.kv);
    if (kv.second.tmap) cudaFree(kv.second.tmap);
  }
  if (st->work) cudaFree(st->work);
  if (st->greedy_logits) cudaFree(st->greedy_logits);
  if (st->wbuf) cudaFree(st->wbuf);
  if (st->err) cudaFree(st->err);
  if (st->ring.host) cudaFreeHost(st->ring.host);
  for (ProfRec& r : st->prof_pending) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  for (cudaEvent_t e : st->ev_pool) cudaEventDestroy(e);
  for (int i = 0; i < RowRing::kEntries; ++i)
    if (st->ring.ev[i]) cudaEventDestroy(st->ring.ev[i]);
  delete st;
  return MG_OK;
}

int mg_stage_memory(const mg_stage* st, uint64_t* wb, uint64_t* kb, uint64_t* xb) {
  if (!st) return fail(MG_EINVAL, "null stage");
  if (wb) *wb = st->wbytes;
  if (kb) *kb = st->kv_bytes;
  if (xb) *xb = st->work_bytes;
  return MG_OK;
}

int mg_kv_alloc(mg_stage* st, int32_t slot, int32_t batch, int32_t capacity) {
  if (!st) return fail(MG_EINVAL, "null stage");
  if (batch < 1 || capacity < 1) return fail(MG_EINVAL, "batch and capacity must be positive");
  if (capacity > st->cfg.max_position_embeddings)
    return fail(MG_EINVAL, "capacity %d exceeds model context %d", capacity,
                st->cfg.max_position_embeddings);
  DeviceGuard guard(st->cfg.device);
  drop_slot(st, slot);
  return reserve_slot(st, slot, batch, capacity, 0);
}

int mg_kv_free(mg_stage* st, int32_t slot) {
  if (!st) return fail(MG_EINVAL, "null stage");
  DeviceGuard guard(st->cfg.device);
  drop_slot(st, slot);
  return MG_OK;
}

int mg_kv_free_all(mg_stage* st) {
  if (!st) return fail(MG_EINVAL, "null stage");
  DeviceGuard guard(st->cfg.device);
  std::vector<int> ids;
  for (auto& kv : st->slots) ids.push_back(kv.first);
  for (int id : ids) drop_slot(st, id);
  return MG_OK;
}

int mg_kv_length(const mg_stage* st, int32_t slot, int32_t* length) {
  if (!st || !length) return fail(MG_EINVAL, "null argument");
  auto it = st->slots.find(slot);
  *length = it == st->slots.end() ? 0 : it->second.len;
  return MG_OK;
}

int mg_kv_batch(const mg_stage* st, int32_t slot, int32_t* batch) {
  if (!st || !batch) return fail(MG_EINVAL, "null argument");
  auto it = st->slots.find(slot);
  *batch = it == st->slots.end() ? 0 : it->second.batch;
  return MG_OK;
}

int mg_kv_trim(mg_stage* st, int32_t slot, int32_t length) {
  if (!st) return fail(MG_EINVAL, "null stage");
  if (length < 0) return fail(MG_EINVAL, "cache length must be non-negative");
  auto it = st->slots.find(slot);
  if (it == st->slots.end() || it->second.len == 0) {
    if (length) return fail(MG_ESTATE, "cannot trim an empty cache to a non-zero length");
    return MG_OK;
  }
  if (it->second.len < length)
    return fail(MG_ESTATE, "cache length %d is shorter than requested %d", it->second.len, length);
  it->second.len = length;
  return MG_OK;
}

int mg_kv_import(mg_stage* st, int32_t slot, int32_t layer, const void* k, const void* v,
                 int32_t length, void* stream) {
  if (!st || !k || !v) return fail(MG_EINVAL, "null argument");
  if (layer < 0 || layer >= st->L) return fail(MG_EINVAL, "local layer %d out of range", layer);
  auto it = st->slots.find(slot);
  if (it == st->slots.end()) return fail(MG_ESTATE, "slot %d does not exist", slot);
  if (length < 0 || length > st->cfg.max_position_embeddings)
    return fail(MG_EINVAL, "length %d outside [0, %d]", length, st->cfg.max_position_embeddings);
  DeviceGuard guard(st->cfg.device);
  cudaStream_t s = (cudaStream_t)stream;
  int rc = reserve_slot(st, slot, it->second.batch, std::max(length, 1), s);
  if (rc) return rc;
  Slot& sl = st->slots[slot];
  MG_LAUNCH(launch_kv_copy(st->cfg.dtype, sl.kv, layer, 0, sl.batch, st->nkv, sl.cap, st->D,
                           length, (void*)k, true, s), "kv import (K)");
  MG_LAUNCH(launch_kv_copy(st->cfg.dtype, sl.kv, layer, 1, sl.batch, st->nkv, sl.cap, st->D,
                           length, (void*)v, true, s), "kv import (V)");
  sl.len = length;
  return MG_OK;
}

int mg_kv_export(const mg_stage* st, int32_t slot, int32_t layer, void* k, void* v, void* stream) {
  if (!st || !k || !v) return fail(MG_EINVAL, "null argument");
  if (layer < 0 || layer >= st->L) return fail(MG_EINVAL, "local layer %d out of range", layer);
  auto it = st->slots.find(slot);
  if (it == st->slots.end()) return fail(MG_ESTATE, "slot %d does not exist", slot);
  DeviceGuard guard(st->cfg.device);
  const Slot& sl = it->second;
  cudaStream_t s = (cudaStream_t)stream;
  MG_LAUNCH(launch_kv_copy(st->cfg.dtype, sl.kv, layer, 0, sl.batch, st->nkv, sl.cap, st->D,
                           sl.len, k, false, s), "kv export (K)");
  MG_LAUNCH(launch_kv_copy(st->cfg.dtype, sl.kv, layer, 1, sl.batch, st->nkv, sl.cap, st->D,
                           sl.len, v, false, s), "kv export (V)");
  return MG_OK;
}

int mg_stage_forward(mg_stage* st, int32_t slot, const int64_t* ids, const void* hidden_in,
                     const int64_t* positions, int32_t batch, int32_t seq, int32_t out_mode,
                     void* out, void* stream) {
  if (!st || !out) return fail(MG_EINVAL, "null argument");
  if (batch < 1 || seq < 1)
    return fail(MG_EINVAL, "input must have shape [batch, sequence] and be non-empty");
  int rc = check_inputs(st, ids, hidden_in);
  if (rc) return rc;
  rc = check_out_mode(st, out_mode);
  if (rc) return rc;
  DeviceGuard guard(st->cfg.device);
  cudaStream_t s = (cudaStream_t)stream;
  auto it = st->slots.find(slot);
  int past = 0;
  if (it != st->slots.end()) {
    if (it->second.batch != batch && it->second.len > 0)
      return fail(MG_EINVAL, "KV cache shape does not match model configuration "
                             "(slot holds %d rows, input has %d)", it->second.batch, batch);
    if (it->second.batch != batch) drop_slot(st, slot);
    else past = it->second.len;
  }
  if (past + seq > st->cfg.max_position_embeddings)
    return fail(MG_EINVAL, "sequence would reach %d positions, but model context is %d",
                past + seq, st->cfg.max_position_embeddings);
  rc = reserve_slot(st, slot, batch, past + seq, s);
  if (rc) return rc;
  Slot& sl = st->slots[slot];
  std::vector<RowDesc> rows(batch);
  for (int b = 0; b < batch; ++b)
    rows[b] = RowDesc{(uint64_t)sl.kv, (uint64_t)sl.tmap, sl.batch, b, sl.cap, past};
  rc = run_stage(st, rows, seq, ids, hidden_in, positions, out_mode, out, s);
  if (rc) return rc;
  sl.len = past + seq;
  return MG_OK;
}

namespace {

int decode_slots(mg_stage* st, const int32_t* slots, int32_t n_slots, const int64_t* ids,
                 const void* hidden_in, int32_t out_mode, void* out, int64_t* greedy_ids, void* stream,
                 const TopPSel* tp = nullptr) {
  int rc = check_inputs(st, ids, hidden_in);
  if (rc) return rc;
  rc = check_out_mode(st, out_mode);
  if (rc) return rc;
  DeviceGuard guard(st->cfg.device);
  cudaStream_t s = (cudaStream_t)stream;
  for (int i = 0; i < n_slots; ++i)
    for (int j = 0; j < i; ++j)
      if (slots[i] == slots[j]) return fail(MG_EINVAL, "slot %d listed twice", slots[i]);
  std::vector<RowDesc> rows;
  for (int i = 0; i < n_slots; ++i) {
    auto it = st->slots.find(slots[i]);
    if (it == st->slots.end() || it->second.len == 0)
      return fail(MG_ESTATE, "slot %d has no cached prefix", slots[i]);
    const int past = it->second.len;
    if (past + 1 > st->cfg.max_position_embeddings)
      return fail(MG_EINVAL, "sequence would reach %d positions, but model context is %d",
                  past + 1, st->cfg.max_position_embeddings);
    rc = reserve_slot(st, slots[i], it->second.batch, past + 1, s);
    if (rc) return rc;
  }
  for (int i = 0; i < n_slots; ++i) {
    const Slot& sl = st->slots[slots[i]];
    for (int b = 0; b < sl.batch; ++b)
      rows.push_back(RowDesc{(uint64_t)sl.kv, (uint64_t)sl.tmap, sl.batch, b, sl.cap, sl.len});
  }
  rc = run_stage(st, rows, 1, ids, hidden_in, nullptr, out_mode, out, s, greedy_ids, tp);
  if (rc) return rc;
  for (int i = 0; i < n_slots; ++i) st->slots[slots[i]].len += 1;
  return MG_OK;
}

}  // namespace

int mg_stage_decode_multi(mg_stage* st, const int32_t* slots, int32_t n_slots, const int64_t* ids,
                          const void* hidden_in, int32_t out_mode, void* out, void* stream) {
  if (!st || !slots || n_slots < 1 || !out) return fail(MG_EINVAL, "null or empty argument");
  return decode_slots(st, slots, n_slots, ids, hidden_in, out_mode, out, nullptr, stream);
}

int mg_stage_decode_greedy(mg_stage* st, const int32_t* slots, int32_t n_slots, const int64_t* ids,
                           const void* hidden_in, int64_t* ids_out, void* logits_out, void* stream) {
  if (!st || !slots || n_slots < 1 || !ids_out) return fail(MG_EINVAL, "null or empty argument");
  if (!st->cfg.has_lm_head) return fail(MG_EINVAL, "greedy selection needs the last stage (lm_head)");
  return decode_slots(st, slots, n_slots, ids, hidden_in, MG_OUT_LOGITS_ALL, logits_out, ids_out, stream);
}

int mg_stage_weight(const mg_stage* st, int32_t which, int32_t layer, void** ptr) {
  if (!st || !ptr) return fail(MG_EINVAL, "null argument");
  *ptr = nullptr;
  const bool per_layer = which >= MG_W_INPUT_NORM && which <= MG_W_DOWN;
  if (per_layer && (layer < 0 || layer >= (int)st->layers.size()))
    return fail(MG_EINVAL, "local layer %d outside [0, %d)", layer, (int)st->layers.size());
  switch (which) {
    case MG_W_EMBED: *ptr = st->embed; break;
    case MG_W_NORM: *ptr = st->norm; break;
    case MG_W_LM_HEAD: *ptr = st->lm_head; break;
    case MG_W_INPUT_NORM: *ptr = st->layers[layer].ln1; break;
    case MG_W_QKV: *ptr = st->layers[layer].wqkv; break;
    case MG_W_Q_NORM: *ptr = st->layers[layer].qn; break;
    case MG_W_K_NORM: *ptr = st->layers[layer].kn; break;
    case MG_W_O: *ptr = st->layers[layer].wo; break;
    case MG_W_POST_NORM: *ptr = st->layers[layer].ln2; break;
    case MG_W_GATE_UP: *ptr = st->layers[layer].wgu; break;
    case MG_W_DOWN: *ptr = st->layers[layer].wd; break;
    default: return fail(MG_EINVAL, "unknown weight %d", which);
  }
  return MG_OK;
}

int mg_stage_probe_wait(mg_stage* st, uint32_t limit_us, int32_t flag_set, void* stream) {
  if (!st) return fail(MG_EINVAL, "null stage");
  if (limit_us < 1 || limit_us > 2000000u) return fail(MG_EINVAL, "limit_us must be in [1, 2000000]");
  DeviceGuard guard(st->cfg.device);
  cudaStream_t s = (cudaStream_t)stream;
  int* flag = st->err + 1;
  MG_CUDA(cudaMemsetAsync(flag, flag_set ? 0x01 : 0, sizeof(int), s), "probe flag");
  MG_LAUNCH(launch_wait_probe(flag, (uint64_t)limit_us * 1000ull, st->err, s), "wait probe");
  MG_CUDA(cudaMemsetAsync(flag, 0, sizeof(int), s), "probe flag reset");
  return MG_OK;
}

int mg_stage_decode_top_p(mg_stage* st, const int32_t* slots, int32_t n_slots, const int64_t* ids,
                          const void* hidden_in, float temperature, float top_p, const float* uniforms,
                          int64_t* ids_out, void* logits_out, void* stream) {
  if (!st || !slots || n_slots < 1 || !ids_out || !logits_out)
    return fail(MG_EINVAL, "null or empty argument");
  if (!st->cfg.has_lm_head) return fail(MG_EINVAL, "top-p selection needs the last stage (lm_head)");
  if (!(temperature > 0.f) || temperature != temperature || temperature > 3.4e38f)
    return fail(MG_EINVAL, "temperature must be a finite positive number");
  if (!(top_p >= 0.f && top_p <= 1.f)) return fail(MG_EINVAL, "top_p must be a finite number in [0, 1]");
  if (!uniforms) return fail(MG_EINVAL, "uniforms are required");
  const TopPSel tp{temperature, top_p, uniforms, ids_out};
  return decode_slots(st, slots, n_slots, ids, hidden_in, MG_OUT_LOGITS_ALL, logits_out, nullptr, stream, &tp);
}

int mg_stage_check_device(mg_stage* st, void* stream) {
  if (!st) return fail(MG_EINVAL, "null stage");
  DeviceGuard guard(st->cfg.device);
  int h = 0;
  MG_CUDA(cudaMemcpyAsync(&h, st->err, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream),
          "error word read");
  MG_CUDA(cudaStreamSynchronize((cudaStream_t)stream), "error word sync");
  if (h == kErrNone) return MG_OK;
  MG_CUDA(cudaMemset(st->err, 0, sizeof(int)), "error word reset");
  if (h == kErrTokenRange)
    return fail(MG_EDEVICE, "input_ids contain a value outside [0, %d)", st->cfg.vocab_size);
  if (h == 3) {
    // A tensor-core kernel gave up waiting for its data; its tile counters
    // may be left mid-count, so clear them before the next forward.
    if (st->counters) cudaMemset(st->counters, 0, st->counters_elems * sizeof(int));
    if (st->greedy_best) cudaMemset(st->greedy_best, 0, 64 * sizeof(unsigned long long));
    return fail(MG_ETIMEOUT, "a kernel gave up a bounded wait (code 3); the outputs of the "
                             "forwards since the last check are invalid");
  }
  return fail(MG_EDEVICE, "position_ids contain a value outside [0, %d)",
              st->cfg.max_position_embeddings);
}

int mg_stage_profile(mg_stage* st, int32_t enable) {
  if (!st) return fail(MG_EINVAL, "null stage");
  DeviceGuard guard(st->cfg.device);
  int rc = prof_collect(st);
  if (rc) return rc;
  if (enable) st->prof = mg_profile{};
  st->profiling = enable != 0;
  return MG_OK;
}

int mg_stage_profile_read(mg_stage* st, mg_profile* out) {
  if (!st || !out) return fail(MG_EINVAL, "null argument");
  DeviceGuard guard(st->cfg.device);
  int rc = prof_collect(st);
  if (rc) return rc;
  *out = st->prof;
  return MG_OK;
}

uint64_t mg_launch_count(void) { return g_launches.load(); }

uint64_t mg_linear_scratch(int32_t dtype, int32_t M, int32_t N, int32_t K, int32_t epilogue) {
  return linear_scratch_elems(dtype, M, N, K, epilogue);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Error word of the standalone linear entry points (mg_linear and
// mg_linear_noalloc): a bounded wait inside the decode GEMM that runs out
// records code 3 here instead of in a stage's word.  A file-scope device
// array, so it needs no allocation; its address is looked up per device.
// ---------------------------------------------------------------------------
namespace {

static __device__ int g_linear_err;

struct SymbolCache {
  void* ptr[64] = {};
  std::mutex mu;
};

// Device address of `symbol` on the current device.  In host code a
// __device__ variable's name is a host-side stand-in, never device memory, so
// the address must come from cudaGetSymbolAddress.  Looked up again on every
// call outside stream capture (cheap once the module is loaded, and it follows
// a cudaDeviceReset); during capture the last looked-up address is used.
int symbol_address(SymbolCache& cache, const void* symbol, cudaStream_t stream, void** out,
                   const char* what) {
  int dev = -1;
  MG_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(MG_EINVAL, "device ordinal %d out of range", dev);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  MG_CUDA(cudaStreamIsCapturing(stream, &cap), "cudaStreamIsCapturing");
  std::lock_guard<std::mutex> lock(cache.mu);
  if (cap == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    MG_CUDA(cudaGetSymbolAddress(&p, symbol), what);
    cache.ptr[dev] = p;
  } else if (!cache.ptr[dev]) {
    return fail(MG_ESTATE, "%s: make one call on this device before capturing a stream", what);
  }
  *out = cache.ptr[dev];
  return MG_OK;
}

SymbolCache g_linear_err_addr;

}  // namespace

extern "C" {

int mg_linear(int32_t dtype, const void* X, int64_t ldx, const void* W, int32_t M, int32_t N,
              int32_t K, int32_t epilogue, const void* R, int64_t ldr, void* Y, int64_t ldy,
              float* scratch, uint64_t scratch_elems, void* stream) {
  if (!X || !W || !Y || M < 0 || N < 1 || K < 1) return fail(MG_EINVAL, "invalid linear arguments");
  if (dtype != MG_DTYPE_F32 && dtype != MG_DTYPE_BF16) return fail(MG_EINVAL, "invalid dtype");
  if (epilogue < MG_EPI_STORE || epilogue > MG_EPI_SWIGLU) return fail(MG_EINVAL, "invalid epilogue");
  if (epilogue == MG_EPI_RESID && !R) return fail(MG_EINVAL, "the residual epilogue needs R");
  if (ldx < K || ldy < N || (R && ldr < N)) return fail(MG_EINVAL, "leading dimensions too small");
  const int vec = dtype == MG_DTYPE_BF16 ? 8 : 4;
  if (K % vec || N % vec || ldx % vec || ldy % vec || (R && ldr % vec))
    return fail(MG_EINVAL, "K, N and leading dimensions must be multiples of 16 bytes");
  if (linear_scratch_elems(dtype, M, N, K, epilogue) > scratch_elems)
    return fail(MG_EINVAL, "scratch too small: %llu fp32 elements needed",
                (unsigned long long)linear_scratch_elems(dtype, M, N, K, epilogue));
  LinearArgs la{};
  la.dtype = dtype;
  la.X = X; la.ldx = ldx; la.W = W; la.Y = Y; la.ldy = ldy; la.R = R; la.ldr = ldr;
  la.M = M; la.N = N; la.K = K; la.epilogue = epilogue;
  la.partial = scratch;
  la.partial_elems = scratch_elems;
  void* err = nullptr;
  int rc = symbol_address(g_linear_err_addr, (const void*)&g_linear_err, (cudaStream_t)stream, &err,
                          "cudaGetSymbolAddress(linear error word)");
  if (rc) return rc;
  la.err = (int*)err;
  MG_LAUNCH(launch_linear(la, (cudaStream_t)stream), "linear");
  return MG_OK;
}

int mg_linear_check_device(void* stream) {
  void* err = nullptr;
  int rc = symbol_address(g_linear_err_addr, (const void*)&g_linear_err, (cudaStream_t)stream, &err,
                          "cudaGetSymbolAddress(linear error word)");
  if (rc) return rc;
  int h = 0;
  MG_CUDA(cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream),
          "linear error word read");
  MG_CUDA(cudaStreamSynchronize((cudaStream_t)stream), "linear error word sync");
  if (h == kErrNone) return MG_OK;
  MG_CUDA(cudaMemset(err, 0, sizeof(int)), "linear error word reset");
  return fail(MG_ETIMEOUT, "a linear launch gave up waiting for its data (code %d); its output is invalid", h);
}

int mg_reserve_sms(int32_t device, int32_t n) {
  int count = 0;
  if (device < 0 || device >= 64) return fail(MG_EINVAL, "device ordinal %d out of range", device);
  MG_CUDA(cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device), "SM count");
  if (n < 0 || n > count / 2) return fail(MG_EINVAL, "reserve between 0 and %d SMs", count / 2);
  mg::g_reserved_sms[device].store(n);
  return MG_OK;
}

int mg_peer_access(int32_t device, int32_t peer, int32_t* enabled) {
  if (!enabled) return fail(MG_EINVAL, "null argument");
  *enabled = 0;
  if (device == peer) {
    *enabled = 1;
    return MG_OK;
  }
  int can = 0;
  MG_CUDA(cudaDeviceCanAccessPeer(&can, device, peer), "cudaDeviceCanAccessPeer");
  if (!can) return MG_OK;  // copies between the pair stage through the host
  DeviceGuard guard(device);
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();  // clear the (non-sticky) "already enabled" error
  } else if (e != cudaSuccess) {
    return cuda_fail(e, "cudaDeviceEnablePeerAccess");
  }
  *enabled = 1;
  return MG_OK;
}

int mg_peer_copy(void* dst, int32_t dst_device, const void* src, int32_t src_device, uint64_t bytes,
                 void* stream) {
  if ((!dst || !src) && bytes) return fail(MG_EINVAL, "null buffer");
  if (bytes == 0) return MG_OK;
  DeviceGuard guard(src_device);  // the stream belongs to the source device
  MG_CUDA(cudaMemcpyPeerAsync(dst, dst_device, src, src_device, (size_t)bytes, (cudaStream_t)stream),
          "cudaMemcpyPeerAsync");
  return MG_OK;
}

int mg_sample_greedy(const void* logits, int32_t dtype, int32_t rows, int32_t vocab,
                     int64_t row_stride, int64_t* ids, void* stream) {
  if (!logits || !ids || rows < 0 || vocab < 1) return fail(MG_EINVAL, "invalid argument");
  MG_LAUNCH(launch_argmax(dtype, logits, rows, vocab, row_stride, ids, (cudaStream_t)stream),
            "greedy sample");
  return MG_OK;
}

int mg_sample_top_p(const void* logits, int32_t dtype, int32_t rows, int32_t vocab,
                    int64_t row_stride, float temperature, float top_p, const float* uniforms,
                    int64_t* ids, void* stream) {
  if (!logits || !ids || rows < 0 || vocab < 1) return fail(MG_EINVAL, "invalid argument");
  if (!(temperature >= 0.f) || temperature != temperature)
    return fail(MG_EINVAL, "temperature must be a finite non-negative number");
  if (!(top_p >= 0.f && top_p <= 1.f)) return fail(MG_EINVAL, "top_p must be a finite number in [0, 1]");
  if (temperature > 0.f && !uniforms) return fail(MG_EINVAL, "uniforms are required");
  MG_LAUNCH(launch_top_p(dtype, logits, rows, vocab, row_stride, temperature, top_p, uniforms, ids,
                         (cudaStream_t)stream),
            "top-p sample");
  return MG_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// mg_linear without allocation: the split-K scratch is a fixed array in the
// library instead of caller- or stage-owned memory.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratch = MG_LINEAR_NOALLOC_SCRATCH;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratch];

// Device address of this process's copy of the array on the current device
// (symbol_address: looked up again outside stream capture).
SymbolCache g_noalloc_addr;

}  // namespace

extern "C" int mg_linear_noalloc(int32_t dtype, const void* X, int64_t ldx, const void* W,
                                 int32_t M, int32_t N, int32_t K, int32_t epilogue, const void* R,
                                 int64_t ldr, void* Y, int64_t ldy, void* stream) {
  if (M < 0 || N < 1 || K < 1) return fail(MG_EINVAL, "invalid linear arguments");
  const uint64_t need = linear_scratch_elems(dtype, M, N, K, epilogue);
  if (need > kNoAllocScratch)
    return fail(MG_EINVAL,
                "this shape needs %llu fp32 elements of split-K scratch; mg_linear_noalloc holds "
                "%llu (use mg_linear with caller scratch)",
                (unsigned long long)need, (unsigned long long)kNoAllocScratch);
  void* scratch = nullptr;
  int rc = symbol_address(g_noalloc_addr, (const void*)g_noalloc_scratch, (cudaStream_t)stream, &scratch,
                          "cudaGetSymbolAddress(noalloc scratch)");
  if (rc) return rc;
  return mg_linear(dtype, X, ldx, W, M, N, K, epilogue, R, ldr, Y, ldy, (float*)scratch,
                   kNoAllocScratch, stream);
}
