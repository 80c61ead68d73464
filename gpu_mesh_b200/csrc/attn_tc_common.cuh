// Device helpers shared by the decode and prefill attention kernels on the
// tensor cores: the visible-key rule, TMA / bulk loads, ldmatrix, the
// m16n8k16 MMA, bf16 packing and the 128-byte swizzle of a K/V box.
#pragma once

#include "kernels.h"
#include "tc_common.cuh"

namespace mg {
namespace attn {

using tc::smem_u32;

// Keys row m (query s of its row, cache row `rd`) may see, following
// LlamaStage's mask policy (models/llama_dense.py:497-532) and HF's cache
// mask for Qwen3.
__device__ __forceinline__ int visible(const AttnArgs& a, const RowDesc& rd, int m, int s) {
  const int total = rd.past + a.S;
  if (a.mask == kMaskSdpa && a.S == 1) return total;
  if (a.mask == kMaskCacheCausal) return min(rd.past + s + 1, total);
  int64_t pos = a.positions ? a.positions[m] : (int64_t)(rd.past + s);
  if (pos < 0) pos = 0;
  return (int)(pos + 1 < (int64_t)total ? pos + 1 : (int64_t)total);
}

// Query tiles of the prefill kernels: a work item is (cache row, KV head,
// tile of tq = 128 / G tokens x the G heads sharing the KV head), heaviest
// (latest) tiles first.
struct PrefillPlan {
  int tq;      // tokens of a tile (128 / G)
  int ntiles;  // query tiles per cache row
  long long items;
};

// Item i (heaviest first): query tile, cache row, KV head.
__device__ __forceinline__ void item_of(const AttnArgs& a, const PrefillPlan& pl, long long i, int& qt, int& b,
                                        int& h) {
  const long long bh = (long long)a.B * a.nkv;
  qt = pl.ntiles - 1 - (int)(i / bh);
  const int rem = (int)(i % bh);
  b = rem / a.nkv;
  h = rem % a.nkv;
}

// The most keys any token of the tile sees: the item's chunk count follows
// from it.  Without explicit positions a token sees min(past + s + 1, total)
// keys (or all of them), which never decreases with s, so the tile's last
// token decides; explicit positions can be in any order, so every token is
// asked.  (Every role evaluates this at each work item's start, where the
// per-token loop cost about 2000 cycles of the item boundary.)
__device__ __forceinline__ int tile_keys(const AttnArgs& a, const RowDesc& rd, const PrefillPlan& pl, int b,
                                         int qt) {
  int s_hi = (qt + 1) * pl.tq;
  if (s_hi > a.S) s_hi = a.S;
  if (s_hi <= qt * pl.tq) return 0;
  if (a.positions == nullptr) return visible(a, rd, b * a.S + s_hi - 1, s_hi - 1);
  int kmax = 0;
  for (int s = qt * pl.tq; s < s_hi; ++s) kmax = max(kmax, visible(a, rd, b * a.S + s, s));
  return kmax;
}

__device__ __forceinline__ void tma_load_2d_gmap(void* dst, uint64_t tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  // rows 8-15 of A (heads >= 8) are zero: a1 = a3 = 0
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const uint32_t a = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t b = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return a | (b << 16);
}

// The two bf16 halves of a packed pair, widened.
__device__ __forceinline__ float lo_bf16(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float hi_bf16(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Byte offset of (key row r, 16-byte chunk c of 64 dims) inside a swizzled box.
__device__ __forceinline__ uint32_t swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// The full m16n8k16 MMA (rows g and g + 8 of A in a0/a2 and a1/a3).
__device__ __forceinline__ void mma16816_full(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Transpose of an 8x8 matrix of 16-bit values held one bf16 pair per thread
// (row lane / 4, columns 2 (lane % 4), + 1).
__device__ __forceinline__ uint32_t movm_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

}  // namespace attn
}  // namespace mg
