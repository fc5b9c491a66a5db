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

}  // namespace

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
