// fa4d_mask.cu — block-occupancy pre-pass over a 4D bool mask.
//
// The reference's kernels visit every 128-key tile of every query block and apply
// the mask element by element (python/fa2.py:95-124 forward, :242-302 backward),
// so a packed-document mask whose tiles are mostly False costs as much as a dense
// one.  This pass reads the mask once and classifies each 128 x 128 block as
// EMPTY (no True element), FULL (every in-bounds element True) or PARTIAL.  The
// forward and backward kernels then skip EMPTY blocks and skip the mask loads of
// FULL ones.  Elements past Tq / Tk do not affect the state of an edge block.
//
// Grid: (ceil(Tk / 512), ceil(Tq / 128), Bm * Hm); 256 threads.  Warp w reads rows
// w, w+8, ... of the CTA's 128-row block; lane l covers 16 consecutive keys, so a
// warp covers 512 keys = 4 blocks and lanes 8j..8j+7 cover block j.
#include "fa4d_kernels.h"
#include "fa4d_ptx.cuh"

namespace fa4d {

namespace {

// True when no byte of w is zero.
__device__ __forceinline__ bool no_zero_byte(uint32_t w) { return ((w - 0x01010101u) & ~w & 0x80808080u) == 0u; }

template <bool kVec>
__global__ void __launch_bounds__(256) mask_blocks_kernel(const MaskBlocksParams p) {
  __shared__ uint32_t s_any[4], s_all[4];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int bh = blockIdx.z;
  const int b = bh / p.Hm;
  const int h = bh - b * p.Hm;
  const int qb = blockIdx.y;
  const int c0 = blockIdx.x * 512 + 16 * lane;
  if (tid < 4) {
    s_any[tid] = 0u;
    s_all[tid] = 1u;
  }
  __syncthreads();

  const uint8_t* base = p.mask + b * p.stride[0] + h * p.stride[1];
  const int r_end = min(qb * 128 + 128, p.Tq);
  bool any = false, all = true;
  if (kVec) {
    // Tk is a multiple of 16 here, so a lane's 16 keys are all in or all out of bounds.
    if (c0 < p.Tk) {
#pragma unroll 4
      for (int r = qb * 128 + warp; r < r_end; r += 8) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(base + static_cast<int64_t>(r) * p.stride[2] + c0));
        any = any || ((w.x | w.y | w.z | w.w) != 0u);
        all = all && no_zero_byte(w.x) && no_zero_byte(w.y) && no_zero_byte(w.z) && no_zero_byte(w.w);
      }
    }
  } else {
    for (int r = qb * 128 + warp; r < r_end; r += 8) {
      const uint8_t* row = base + static_cast<int64_t>(r) * p.stride[2];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        if (c0 + e < p.Tk) {
          const bool keep = __ldg(row + c0 + e) != 0;
          any = any || keep;
          all = all && keep;
        }
      }
    }
  }
  const uint32_t any_b = __ballot_sync(0xffffffffu, any);
  const uint32_t all_b = __ballot_sync(0xffffffffu, all);
  if (lane < 4) {
    if ((any_b >> (8 * lane)) & 0xFFu) atomicOr(&s_any[lane], 1u);
    if (((all_b >> (8 * lane)) & 0xFFu) != 0xFFu) atomicAnd(&s_all[lane], 0u);
  }
  __syncthreads();
  if (tid < 4) {
    const int kb = blockIdx.x * 4 + tid;
    if (kb < p.nkb) {
      const uint8_t state = s_any[tid] ? (s_all[tid] ? 2 : 1) : 0;
      p.blocks[(static_cast<int64_t>(bh) * p.nqb + qb) * p.nkb + kb] = state;
    }
  }
}

// Keep flags of 32 consecutive bytes as one word (bit j = byte j nonzero).
__device__ __forceinline__ uint32_t keep_word(const uint4& a, const uint4& b) {
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t r = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) r |= keep_bits4(w[i]) << (4 * i);
  return r;
}

// One pass over the mask writes, for every 128 x 128 block, its state, plus the mask
// as packed bits in the two tile layouts the kernels read with one vector load per
// thread and tile:
//   row bits [Bm*Hm][nkb][Tq][4] words: 128 keys of key tile kt for query row q
//     (bit j of word w = key 128*kt + 32*w + j), read by the forward;
//   column bits [Bm*Hm][nqt][Tk][2] words: 64 queries of query tile qt for key k
//     (bit j of word w = query 64*qt + 32*w + j), read by the backward.
// Keys / queries past Tk / Tq read as 0.  Grid: (ceil(Tk / 512), ceil(Tq / 128),
// Bm * Hm), 128 threads; warp w owns query rows 32w..32w+31 of the block row
// (lane = row) and walks 16 chunks of 32 keys; column words come from one ballot per key.
// Source of the keep flags: mask bytes (kVec: 16-byte loads) or per-token document
// ids (kDocs: keep iff the query's and the key's ids are equal and not negative).
template <bool kVec, bool kDocs>
__global__ void __launch_bounds__(128) mask_prepare_kernel(const MaskPrepParams p) {
  __shared__ uint32_t s_any[4], s_all[4];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int bh = blockIdx.z;
  const int b = bh / p.Hm;
  const int h = bh - b * p.Hm;
  const int qb = blockIdx.y;
  const int q0w = qb * 128 + 32 * warp;  // first row of this warp
  const int row = q0w + lane;
  const bool row_ok = row < p.Tq;
  if (tid < 4) {
    s_any[tid] = 0u;
    s_all[tid] = 1u;
  }
  __syncthreads();
  const uint8_t* src = kDocs ? nullptr
                             : p.mask + b * p.stride[0] + h * p.stride[1] +
                                   static_cast<int64_t>(row_ok ? row : 0) * p.stride[2];
  const int32_t doc_row = (kDocs && row_ok) ? __ldg(p.doc_q + b * p.doc_q_stride + row) : -1;
  uint32_t* row_bits = p.row_bits + static_cast<int64_t>(bh) * p.nkb * p.Tq * 4;
  // This warp's 32 rows are half (q0w / 32) % 2 of query tile q0w / 64.
  const int qt = q0w >> 6;
  const bool col_ok = qt < p.nqt;
  uint32_t* col_bits = p.col_bits + (static_cast<int64_t>(bh) * p.nqt + qt) * p.Tk * 2 + ((q0w >> 5) & 1);
  bool any_blk = false, all_blk = true;
#pragma unroll 1
  for (int it = 0; it < 16; ++it) {
    const int kc = blockIdx.x * 512 + 32 * it;
    // Keys of this chunk inside Tk (as bits).
    const int nin = min(max(p.Tk - kc, 0), 32);
    const uint32_t inb = nin >= 32 ? 0xffffffffu : ((1u << nin) - 1u);
    uint32_t rw = 0u;
    if (kDocs) {
      // Lane j holds key kc+j's document; each row compares against all 32.
      const int32_t doc_key = (kc + lane < p.Tk) ? __ldg(p.doc_k + b * p.doc_k_stride + kc + lane) : -2;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int32_t dk = __shfl_sync(0xffffffffu, doc_key, j);
        if (doc_row >= 0 && dk == doc_row) rw |= 1u << j;
      }
    } else if (row_ok && nin > 0) {
      if (kVec) {
        // Tk % 16 == 0: each 16-byte half is entirely in or out of bounds.
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(src + kc));
        const uint4 c = nin > 16 ? __ldg(reinterpret_cast<const uint4*>(src + kc + 16)) : z;
        rw = keep_word(a, c);
      } else {
#pragma unroll 4
        for (int j = 0; j < 32; ++j)
          if (j < nin && __ldg(src + kc + j) != 0) rw |= 1u << j;
      }
    }
    rw &= inb;
    const int kt = kc >> 7;
    if (row_ok && kt < p.nkb) row_bits[(static_cast<int64_t>(kt) * p.Tq + row) * 4 + ((kc >> 5) & 3)] = rw;
    // Column words: bit `lane` of the ballot for key kc+j is row q0w+lane's flag.
    uint32_t mine = 0u;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const uint32_t bal = __ballot_sync(0xffffffffu, (rw >> j) & 1u);
      if (lane == j) mine = bal;
    }
    if (kc + lane < p.Tk && col_ok) col_bits[static_cast<int64_t>(kc + lane) * 2] = mine;
    any_blk = any_blk || __any_sync(0xffffffffu, rw != 0u);
    all_blk = all_blk && __all_sync(0xffffffffu, !row_ok || rw == inb);
    if ((it & 3) == 3) {
      if (lane == 0) {
        if (any_blk) atomicOr(&s_any[it >> 2], 1u);
        if (!all_blk) atomicAnd(&s_all[it >> 2], 0u);
      }
      any_blk = false;
      all_blk = true;
    }
  }
  __syncthreads();
  if (tid < 4) {
    const int kb = blockIdx.x * 4 + tid;
    if (kb < p.nkb) {
      const uint8_t state = s_any[tid] ? (s_all[tid] ? 2 : 1) : 0;
      p.blocks[(static_cast<int64_t>(bh) * p.nqb + qb) * p.nkb + kb] = state;
    }
  }
}

}  // namespace

cudaError_t launch_mask_prepare(const MaskPrepParams& p, cudaStream_t s) {
  dim3 grid((p.Tk + 511) / 512, p.nqb, p.Bm * p.Hm);
  if (p.doc_q)
    mask_prepare_kernel<false, true><<<grid, 128, 0, s>>>(p);
  else if (p.vec)
    mask_prepare_kernel<true, false><<<grid, 128, 0, s>>>(p);
  else
    mask_prepare_kernel<false, false><<<grid, 128, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_mask_blocks(const MaskBlocksParams& p, cudaStream_t s) {
  const bool vec = p.vec != 0;
  dim3 grid((p.Tk + 511) / 512, p.nqb, p.Bm * p.Hm);
  if (vec)
    mask_blocks_kernel<true><<<grid, 256, 0, s>>>(p);
  else
    mask_blocks_kernel<false><<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace fa4d
