// fa4d_tiles.cuh — which 128-key tiles a 128-row query tile visits (key bound, causal
// limit, EMPTY blocks of the mask's block map) and the keep bits of a mask row read as
// bytes; shared by the forward and the deterministic dQ kernels; and the (query head,
// 64-row query tile) pairs a 128-key tile of the backward visits.
#pragma once

#include <cstdint>

#include "fa4d_ptx.cuh"

namespace fa4d {

// Number of 128-key tiles query rows [qs, qe) need (0 if qs >= Tq); with `causal`,
// key k is kept for query q iff k <= q + causal_off.
__device__ __forceinline__ int kv_tile_count(int qs, int qe, int Tq, int Tk, int causal, int causal_off) {
  if (qs >= Tq) return 0;
  int kv_end = Tk;
  if (causal) {
    const long long lim = static_cast<long long>(qe) + causal_off;  // keys < qe + off
    kv_end = lim < Tk ? static_cast<int>(lim) : Tk;
  }
  return kv_end > 0 ? (kv_end + 127) / 128 : 0;
}

// The 128-key tiles one 128-row query slot visits: the tiles below n (key bounds and
// the causal limit) minus the EMPTY blocks of the mask's block map.
template <bool kMask>
struct SlotTiles {
  const uint8_t* map;  // this slot's row of the block map, or null
  int n;
  // 0: skip; 1: visit and apply the mask; 2: visit, the mask keeps every key.
  __device__ __forceinline__ int state(int kt) const {
    if (kt >= n) return 0;
    if (!kMask) return 2;
    if (!map) return 1;
    const int v = __ldg(map + kt);
    return v == 0 ? 0 : (v == 2 ? 2 : 1);
  }
  __device__ __forceinline__ int next(int kt) const {
    while (kt < n && state(kt) == 0) ++kt;
    return kt;
  }
  __device__ __forceinline__ int last() const {
    int kt = n - 1;
    while (kt >= 0 && state(kt) == 0) --kt;
    return kt;
  }
};

// The (query head g of the GQA group, 64-row query tile) pairs a key tile visits, in
// order g-major, minus those whose 128 x 128 block the mask's block map marks EMPTY
// (block-sparse skipping; the reference visits every pair, python/fa2.py:242).
template <bool kMask>
struct QTiles {
  const uint8_t* map;  // block map at (head 0 of the group, query block 0, this key block), or null
  int64_t head_stride, row_stride;
  int nq, first_qt, N;  // N = G * nq pairs before skipping
  int lin;              // current pair g * nq + qi; lin >= N past the end
  __device__ __forceinline__ int g() const { return lin / nq; }
  __device__ __forceinline__ int q0() const { return (first_qt + lin % nq) * 64; }
  // 0: skip; 1: visit and apply the mask; 2: visit, the mask keeps every pair.
  __device__ __forceinline__ int state() const {
    if (!kMask) return 2;
    if (!map) return 1;
    const int gg = lin / nq;
    const int v = __ldg(map + gg * head_stride + ((first_qt + lin - gg * nq) >> 1) * row_stride);
    return v == 0 ? 0 : (v == 2 ? 2 : 1);
  }
  __device__ __forceinline__ bool valid() const { return lin < N; }
  __device__ __forceinline__ void skip_empty() {
    if (kMask && map)
      while (lin < N && state() == 0) ++lin;
  }
  __device__ __forceinline__ void advance() {
    ++lin;
    skip_empty();
  }
};

// Keep bits of keys kbase..kbase+127 of one mask row read as bytes (the path without
// prepared bits).  Kept out of line so its loads do not raise the register pressure
// of the softmax loop.
static __device__ __noinline__ uint4 mask_words_from_bytes(const uint8_t* row, int kbase, int Tk, int vec) {
  uint32_t w[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int kc = kbase + 32 * c;
    uint32_t x = 0u;
    // kc is the same for every lane, so these branches are warp-uniform.
    if (vec && kc + 31 < Tk) {
#pragma unroll
      for (int u = 0; u < 8; ++u) x |= keep_bits4(__ldg(reinterpret_cast<const unsigned int*>(row + kc) + u)) << (4 * u);
    } else {
      for (int e = 0; e < 32; ++e)
        if (kc + e < Tk) x |= (__ldg(row + kc + e) != 0 ? 1u : 0u) << e;
    }
    w[c] = x;
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

}  // namespace fa4d
