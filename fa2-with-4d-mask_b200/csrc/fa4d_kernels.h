// fa4d_kernels.h — parameter blocks handed to the sm_100a kernels and the launch
// entry points the C ABI (fa4d_api.cu) dispatches to.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace fa4d {

// Forward: one CTA owns 2 x 128 query rows of one (batch, query head) and streams
// the key/value tiles of the matching KV head.
struct FwdParams {
  CUtensorMap tm_q;  // dims (D, Tq, Hq, B), box (64, 128, 1, 1), 128-B swizzle
  CUtensorMap tm_k;  // dims (D, Tk, Hk, B), box (64, 128, 1, 1)
  CUtensorMap tm_v;
  void* o;
  float* lse;
  const uint8_t* mask;
  const float* score;
  int64_t o_stride[3];      // (b, t, h) elements
  int64_t mask_stride[3];   // (b, h, row) elements
  int64_t score_stride[3];
  int32_t B, Tq, Tk, Hq, Hk;
  int32_t lse_ld;           // LSE row stride (floats)
  int32_t causal;           // 0 / 1 (a causal mode is on)
  int32_t causal_off;       // key k is kept for query q iff k <= q + causal_off
  float scale_log2;         // scale * log2(e)
  int32_t mask_vec;         // 1: rows are 4-B aligned, 32-bit loads allowed
  int32_t score_vec;        // 1: rows are 16-B aligned, 128-bit loads allowed
  int* status;              // device status word (bounded-wait timeouts)
  // Block map (fa4d_mask_blocks) or null: byte b*mb_stride[0] + h*mb_stride[1] +
  // qb*nkb + kb holds the state of the 128 x 128 block (qb, kb).
  const uint8_t* mask_blocks;
  int64_t mb_stride[2];
  int32_t nkb;
  // bias_tma = 1: mask / score tiles are staged in shared memory by TMA through
  // these maps (dims (Tk, Tq, H or 1, B or 1); mask box (128, 128), score box
  // (32, 128), 128-B swizzle); 0: the softmax threads load them from global memory.
  int32_t bias_tma;
  CUtensorMap tm_mask;
  CUtensorMap tm_score;
  // Prepared row bits (fa4d_mask_prepare) or null: the uint4 at word offset
  // b*mbits_stride[0] + h*mbits_stride[1] + (kt*Tq + q)*4 holds the keep flags of
  // the 128 keys of key tile kt for query row q.
  const uint32_t* mask_bits;
  int64_t mbits_stride[2];
  // 1: rows that keep no key get O = 0 instead of NaN (document-id mode, where such
  // rows are padding).
  int32_t empty_rows_zero;
  // Head dim of the tensors (<= the kernel's compute width D; the tensor maps zero-fill
  // columns d_out..D-1, so those columns compute zeros and are not stored).
  int32_t d_out;
};

// Backward: one CTA owns 128 keys of one (batch, KV head), loops over every
// query head of the GQA group and every 64-row query tile, accumulates dK/dV in
// tensor memory and adds dQ into an fp32 accumulator.
struct BwdParams {
  CUtensorMap tm_q;   // dims (D, Tq, Hq, B), box (64, 64, 1, 1)
  CUtensorMap tm_do;  // same for dO
  CUtensorMap tm_k;   // dims (D, Tk, Hk, B), box (64, 128, 1, 1)
  CUtensorMap tm_v;
  const float* lse;     // [B, Hq, lse_ld]
  const float* delta;   // [B, Hq, lse_ld]
  float* dq_acc;        // [B, Hq, lse_ld, D] fp32, zeroed by the preprocess kernel
  void* dk;
  void* dv;
  const uint8_t* mask;
  const float* score;
  int64_t dk_stride[3];
  int64_t dv_stride[3];
  int64_t mask_stride[3];
  int64_t score_stride[3];
  int32_t B, Tq, Tk, Hq, Hk;
  int32_t lse_ld;
  int32_t causal;
  int32_t causal_off;
  float scale_log2;
  float scale;
  int* status;
  const uint8_t* mask_blocks;  // as in FwdParams
  int64_t mb_stride[2];
  int32_t nkb;
  // Prepared column bits or null: the uint2 at word offset b*mbt_stride[0] +
  // h*mbt_stride[1] + (qt*Tk + k)*2 holds the keep flags of the 64 queries of
  // query tile qt for key k.
  const uint32_t* mask_bits_t;
  int64_t mbt_stride[2];
  // score_pf = 1: the producer prefetches each query tile's score into L2 through
  // tm_score (dims (Tk, Tq, H or 1, B or 1), box (32, 64)).
  int32_t score_pf;
  CUtensorMap tm_score;
  // Group split: g_split CTAs share one key tile, each taking Hq/Hk/g_split query heads
  // of the group; with g_split > 1 each writes its fp32 partial dK, dV into slice
  // `split` of [g_split][B, Tk, Hk, D] (part_stride elements per slice) instead of dk / dv.
  int32_t g_split;
  float* dk_part;
  float* dv_part;
  int64_t part_stride;
  // 1: dQ is computed by dq_kernel (deterministic mode); this kernel skips its dQ
  // products and the drain.
  int32_t skip_dq;
  int32_t d_out;  // head dim of dK / dV (as in FwdParams); dq_acc and the slices use D
  // 1: grid (key tiles, KV head x split, B), key tiles fastest, so a wave covers whole
  // heads and each dQ accumulator tile receives all its key tiles' additions while it
  // is in L2 (equal-work grids); 0: grid (KV head x split, key tiles, B), the longest
  // key tiles first (causal and block-sparse grids).
  int32_t kb_fastest;
  // V itself (16-bit, strides (b, t, h) in elements, rows 16-B aligned): the D = 256
  // kernel copies each key's V row into tensor memory with plain loads.
  const void* v;
  int64_t v_stride[3];
  const void* k;        // D = 256: rank 0 copies its K tile into TMEM (A operand of S^T)
  int64_t k_stride[3];
  // Block-sparse grids with a prepared mask: the key tile of grid row rank comes from
  // kb_order (mask batch / head strides ko_stride, 0 where the mask broadcasts), longest
  // first, and the grid is (KV head x split, key-tile rank x B) with the batch fastest
  // in y, so the longest CTAs of every batch element start first.  Null: grid as above.
  const int32_t* kb_order;
  int64_t ko_stride[2];
};

// Deterministic dQ: one CTA per 128-row query tile of one (batch, head) walks its key
// tiles in order (see fa4d_dq.cu, fa4d_dq256.cu).
struct DqParams {
  CUtensorMap tm_q;   // dims (D, Tq, Hq, B), box (64, 128, 1, 1)
  CUtensorMap tm_do;
  CUtensorMap tm_k;   // dims (D, Tk, Hk, B), box (64, 128, 1, 1); (64, 64, 1, 1) at D = 256
  CUtensorMap tm_v;
  const float* lse;
  const float* delta;
  void* dq;
  int64_t dq_stride[3];
  const uint8_t* mask;
  const float* score;
  int64_t mask_stride[3];
  int64_t score_stride[3];
  const uint8_t* mask_blocks;
  int64_t mb_stride[2];
  int32_t nkb;
  const uint32_t* mask_bits;  // prepared row bits, as in FwdParams
  int64_t mbits_stride[2];
  int32_t mask_vec, score_vec;
  int32_t B, Tq, Tk, Hq, Hk;
  int32_t lse_ld;
  int32_t causal;
  int32_t causal_off;
  float scale_log2;
  float scale;
  int* status;
  int32_t d_out;  // head dim of dQ (as in FwdParams)
};

// dK, dV (input dtype, caller strides) from the split-group partial slices.
struct DkvConvertParams {
  const float* dk_part;
  const float* dv_part;
  int64_t part_stride;
  int32_t n_split;
  void* dk;
  void* dv;
  int64_t dk_stride[3];
  int64_t dv_stride[3];
  int32_t B, Tk, Hk, D;  // D: row length of the slices (the compute width)
  int32_t d_out;         // head dim of dK / dV
};

// Block-occupancy pre-pass: blocks[((b * Hm + h) * nqb + qb) * nkb + kb] =
// 0 (no True element) / 1 (some) / 2 (all in-bounds elements True).
struct MaskBlocksParams {
  const uint8_t* mask;
  int64_t stride[3];  // (b, h, row) elements
  int32_t Bm, Hm, Tq, Tk, nqb, nkb;
  int32_t vec;        // 1: base 16-B aligned and row stride a multiple of 16 with Tk % 16 == 0
  uint8_t* blocks;
};

// Mask preparation: block map as above plus the mask as packed bits, row-major for
// the forward and transposed for the backward (see mask_prepare_kernel).
struct MaskPrepParams {
  const uint8_t* mask;
  int64_t stride[3];
  int32_t Bm, Hm, Tq, Tk, nqb, nkb;
  int32_t vec;
  int32_t nqt;        // ceil(Tq / 64)
  // Document ids instead of mask bytes (doc_q non-null): [Bm][Tq] and [Bm][Tk] int32
  // with batch strides; keep (q, k) iff doc_q == doc_k >= 0.
  const int32_t* doc_q;
  const int32_t* doc_k;
  int64_t doc_q_stride, doc_k_stride;
  uint8_t* blocks;
  uint32_t* row_bits;
  uint32_t* col_bits;
  int32_t* kb_order;  // [Bm * Hm][nkb]: key tiles by live query blocks, most first
};

// Row dot products Delta = rowsum(O * dO) and zeroing of the dQ accumulator.
struct PrepParams {
  const void* o;
  const void* dout;
  float* delta;
  float* dq_acc;
  int64_t o_stride[3];
  int64_t do_stride[3];
  int32_t B, Tq, Hq, D;  // D: row length of dq_acc (the compute width)
  int32_t lse_ld;
  int32_t d_out;         // head dim of O / dO
};

// dQ (input dtype, caller strides) = dQ accumulator [B, Hq, lse_ld, D].
struct ConvertParams {
  const float* dq_acc;
  void* dq;
  int64_t dq_stride[3];
  int32_t B, Tq, Hq, D;  // D: row length of dq_acc (the compute width)
  int32_t lse_ld;
  float scale;
  int32_t d_out;         // head dim of dQ
};

cudaError_t launch_fwd(const FwdParams& p, int D, bool bf16, bool has_mask, bool has_score, cudaStream_t s);
cudaError_t launch_bwd(const BwdParams& p, int D, bool bf16, bool has_mask, bool has_score, cudaStream_t s);
cudaError_t launch_bwd256(const BwdParams& p, bool bf16, bool has_mask, bool has_score, cudaStream_t s);
cudaError_t launch_bwd_prep(const PrepParams& p, bool bf16, cudaStream_t s);
cudaError_t launch_dq_convert(const ConvertParams& p, bool bf16, cudaStream_t s);
cudaError_t launch_dkv_convert(const DkvConvertParams& p, bool bf16, cudaStream_t s);
cudaError_t launch_dq(const DqParams& p, int D, bool bf16, bool has_mask, bool has_score, cudaStream_t s);
cudaError_t launch_dq256(const DqParams& p, bool bf16, bool has_mask, bool has_score, cudaStream_t s);
cudaError_t launch_mask_blocks(const MaskBlocksParams& p, cudaStream_t s);
cudaError_t launch_mask_prepare(const MaskPrepParams& p, cudaStream_t s);
cudaError_t launch_wait_timeout_check(int* status, long long limit, cudaStream_t s);
cudaError_t launch_exp2_check(float* out, int n, float lo, float hi, cudaStream_t s);

}  // namespace fa4d
