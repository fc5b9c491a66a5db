/*
 * fa4d.h — C ABI of the B200 (sm_100a) FlashAttention-2 forward/backward with an
 * optional 4D bool mask and fp32 additive score.
 *
 * Every entry point takes plain device pointers, element strides and sizes; no
 * framework types cross this boundary.  The caller owns every buffer (inputs,
 * outputs, LSE and the backward workspace).  The library keeps no state besides
 * a per-device cache of the driver's tensor-map encoder and a device-side status
 * word that kernels set when a bounded wait gives up.
 *
 * Layout convention (matches the kernels' native layout of the reference,
 * python/fa2.py:38-44): Q/O/dO/dQ are [B, Tq, Hq, D] and K/V/dK/dV are
 * [B, Tk, Hk, D], each described by element strides (batch, seq, head); the
 * head-dim stride must be 1.  A BHSD tensor is passed as its transpose(1, 2)
 * view, so no copy is needed.  mask is bool/uint8 and score is fp32, both
 * [B or 1, Hq or 1, Tq, Tk] given by element strides (batch, head, row); a
 * broadcast dimension may have stride 0; the key stride must be 1.
 *
 * Return value: 0 on success, a negative FA4D_ERR_* code otherwise;
 * fa4d_last_error() gives a message for the calling thread.  All work is
 * enqueued on the given stream (a cudaStream_t, NULL = legacy default stream)
 * and nothing synchronises with the host.
 */
#ifndef FA4D_H_
#define FA4D_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FA4D_ABI_VERSION 2

enum fa4d_dtype { FA4D_BF16 = 0, FA4D_F16 = 1 };

/* Causal alignment.  TOP_LEFT keeps key k for query q when k <= q, which is the
 * reference's is_causal semantics (python/fa2.py:75,95 and
 * benchmark/precision_check.py:164-167).  BOTTOM_RIGHT keeps k <= q + (Tk - Tq). */
enum fa4d_causal { FA4D_CAUSAL_NONE = 0, FA4D_CAUSAL_TOP_LEFT = 1, FA4D_CAUSAL_BOTTOM_RIGHT = 2 };

enum fa4d_status {
  FA4D_OK = 0,
  FA4D_ERR_INVALID = -1,     /* bad pointer, shape, stride or enum value */
  FA4D_ERR_UNSUPPORTED = -2, /* valid but not built: head dim not in {64, 96, 128, 256} */
  FA4D_ERR_CUDA = -3,        /* a CUDA runtime call or kernel launch failed */
  FA4D_ERR_DRIVER = -4,      /* cuTensorMapEncodeTiled unavailable or failed */
  FA4D_ERR_LAYOUT = -5,      /* strides/base not 16-byte aligned for TMA: pass a contiguous copy */
  FA4D_ERR_WORKSPACE = -6    /* workspace missing or smaller than fa4d_bwd_workspace_size() */
};

typedef struct fa4d_fwd_args {
  const void* q;           /* [B, Tq, Hq, D] */
  const void* k;           /* [B, Tk, Hk, D] */
  const void* v;           /* [B, Tk, Hk, D] */
  void* o;                 /* [B, Tq, Hq, D], written */
  float* lse;              /* [B, Hq, fa4d_lse_row_stride(Tq)] fp32, written (log2 domain) */
  const uint8_t* mask;     /* optional, NULL = none; nonzero byte = keep */
  const float* score;      /* optional, NULL = none; added to QK^T before scaling */
  int64_t q_stride[3];     /* element strides (batch, seq, head) */
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  int64_t mask_stride[3];  /* element strides (batch, head, row) */
  int64_t score_stride[3];
  int32_t B, Tq, Tk, Hq, Hk, D;
  int32_t dtype;           /* enum fa4d_dtype */
  int32_t causal;          /* enum fa4d_causal */
  float scale;             /* softmax scale applied to (QK^T + score) */
  int32_t reserved[3];
  /* Optional block map of `mask` from fa4d_mask_blocks (NULL = every block is
   * treated as PARTIAL).  The state of 128 x 128 block (qb, kb) for batch b and
   * query head h is the byte at
   *   mask_blocks + b * mask_blocks_stride[0] + h * mask_blocks_stride[1]
   *               + qb * ceil(Tk / 128) + kb;
   * a stride is 0 where the mask broadcasts.  EMPTY blocks are skipped (their keys
   * contribute nothing) and FULL blocks are processed without reading the mask.
   * Ignored when mask is NULL. */
  const uint8_t* mask_blocks;
  int64_t mask_blocks_stride[2];
  /* Optional output of fa4d_mask_prepare for `mask` (NULL = none), 256-B aligned.
   * It holds the block map and the mask as packed bits; when given, the kernels
   * skip EMPTY blocks and read the bits instead of the mask bytes, and
   * mask_blocks is ignored.  It must have been prepared with Bm = (mask_stride[0]
   * ? B : 1) and Hm = (mask_stride[1] ? Hq : 1) and the same Tq, Tk.  With mask ==
   * NULL it may instead come from fa4d_mask_prepare_docs with Bm = B: the keep flags
   * are then those of the document ids (no mask tensor exists). */
  const void* mask_prepared;
} fa4d_fwd_args;

typedef struct fa4d_bwd_args {
  const void* q;
  const void* k;
  const void* v;
  const void* o;           /* forward output */
  const void* dout;        /* [B, Tq, Hq, D] upstream gradient */
  const float* lse;        /* as written by fa4d_fwd */
  const uint8_t* mask;
  const float* score;
  void* dq;                /* [B, Tq, Hq, D] written, input dtype */
  void* dk;                /* [B, Tk, Hk, D] written, input dtype (sum over the GQA group) */
  void* dv;
  int64_t q_stride[3];
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  int64_t do_stride[3];
  int64_t dq_stride[3];
  int64_t dk_stride[3];
  int64_t dv_stride[3];
  int64_t mask_stride[3];
  int64_t score_stride[3];
  int32_t B, Tq, Tk, Hq, Hk, D;
  int32_t dtype;
  int32_t causal;
  float scale;
  int32_t deterministic;   /* 1: bit-reproducible backward — dQ is computed by a
                            * separate pass (one CTA per query tile walking the key
                            * tiles in order, accumulating in tensor memory) instead
                            * of fp32 additions in arrival order; 0: default */
  void* workspace;         /* device scratch, >= fa4d_bwd_workspace_size() bytes, 256-B aligned */
  size_t workspace_bytes;
  const uint8_t* mask_blocks;      /* optional, as in fa4d_fwd_args */
  int64_t mask_blocks_stride[2];
  const void* mask_prepared;       /* optional, as in fa4d_fwd_args */
} fa4d_bwd_args;

/* Row stride (in floats) of the LSE buffer: Tq rounded up to a multiple of 128.
 * The LSE buffer holds B * Hq * fa4d_lse_row_stride(Tq) floats. */
int64_t fa4d_lse_row_stride(int32_t Tq);

/* Bytes of device scratch fa4d_bwd needs: an fp32 dQ accumulator
 * [B, Hq, fa4d_lse_row_stride(Tq), Dc] and the fp32 row dot products
 * Delta [B, Hq, fa4d_lse_row_stride(Tq)], where Dc is the width the kernels compute
 * at (D, except 128 for D = 96).  At D = 256 there is no accumulator (dQ always comes
 * from the ordered pass, which writes it directly). */
size_t fa4d_bwd_workspace_size(int32_t B, int32_t Tq, int32_t Hq, int32_t D);

/* Workspace bytes including the backward's group-split buffers.  fa4d_bwd may split
 * each KV head's query-head group over S CTAs (S a power of two, at most 8, chosen by
 * fa4d_bwd_group_split from the sizes, the causal mode and the current device's SM
 * count): when one CTA per (key tile, KV head, batch) would leave SMs idle (MQA, short
 * key sequences), or when equal-work CTAs would leave the grid's last wave mostly
 * empty.  Each CTA writes its fp32 partial dK/dV into its own slice and the slices are
 * added in a fixed order, so the result does not depend on scheduling.  The size
 * covers the largest split of any causal mode.  A workspace of
 * fa4d_bwd_workspace_size() bytes (no room for the slices) makes fa4d_bwd run
 * unsplit.  Returns fa4d_bwd_workspace_size() when no split would be used. */
size_t fa4d_bwd_workspace_size_ex(int32_t B, int32_t Tq, int32_t Tk, int32_t Hq, int32_t Hk, int32_t D);

/* The group split S fa4d_bwd uses for these sizes and causal mode on the current
 * device when the workspace has fa4d_bwd_workspace_size_ex() bytes (1: unsplit);
 * 0 for invalid sizes. */
int32_t fa4d_bwd_group_split(int32_t B, int32_t Tq, int32_t Tk, int32_t Hq, int32_t Hk, int32_t D, int32_t causal);

/* Forward: O = softmax(((Q K^T + score) * scale) masked) V and LSE.
 * Replaces the launch of flash_attention_fwd_with_4d_mask at
 * python/fa2.py:474-478 (kernel python/fa2.py:22-139). */
int fa4d_fwd(const fa4d_fwd_args* args, void* stream);

/* Backward: dQ, dK, dV from dO.  Replaces bwd_preprocess plus
 * flash_attention_bwd_with_4d_mask_atomic / _reduce and the host-side casts and
 * sums at python/fa2.py:508-549 (kernels python/fa2.py:142-426). */
int fa4d_bwd(const fa4d_bwd_args* args, void* stream);

/* The three stages fa4d_bwd enqueues, callable one by one (same args, same
 * stream order required: preprocess, main, dq_convert).
 *  - fa4d_bwd_preprocess: Delta = rowsum(O * dO) into the workspace and zeroing
 *    of the fp32 dQ accumulator; replaces bwd_preprocess (python/fa2.py:142-179,
 *    launched at :509-513) and the torch.zeros of dQ at :527 / :540.
 *  - fa4d_bwd_main: dK, dV (written) and dQ (accumulated in the workspace);
 *    replaces flash_attention_bwd_with_4d_mask_atomic (python/fa2.py:182-302,
 *    launched at :530-534) and _reduce (:306-426, launched at :543-547).
 *  - fa4d_bwd_dq_convert: dQ in the input dtype from the accumulator; replaces the
 *    autograd engine's cast of the fp32 dQ the reference returns (:556). */
int fa4d_bwd_preprocess(const fa4d_bwd_args* args, void* stream);
int fa4d_bwd_main(const fa4d_bwd_args* args, void* stream);
int fa4d_bwd_dq_convert(const fa4d_bwd_args* args, void* stream);

/* Backward for callers that cannot allocate device memory — no counterpart in the
 * reference.  Some hosts own only the input and output buffers (a plugin or FFI
 * boundary with no device allocator of its own), or run with device memory fully
 * reserved by another pool, where cudaMalloc would fail and cudaFree would
 * synchronise the device.  This call takes the same arguments as fa4d_bwd but ignores
 * args->workspace / workspace_bytes: the scratch (fp32 dQ accumulator and Delta) is a
 * fixed buffer of FA4D_BWD_NOALLOC_MAX_WORKSPACE bytes inside the library, which every
 * GPU that loads the library keeps until the process exits.  Nothing is allocated.
 *  - The buffer is device memory of the library's code module.  The CUDA runtime
 *    reserves it on a device when it loads that module there: at the first call of
 *    any fa4d entry point on that device under lazy module loading (the CUDA 12
 *    default), or when the library is loaded with CUDA_MODULE_LOADING=EAGER.  A host
 *    whose memory pool reserves all device memory should make one fa4d call per
 *    device before the pool does, or that first call fails with FA4D_ERR_CUDA.
 *  - Problems whose fa4d_bwd_workspace_size() exceeds the buffer are rejected with
 *    FA4D_ERR_WORKSPACE (e.g. B=1, Hq=32, D=128 fits up to Tq = 3968).
 *  - The first call on a device looks up the buffer's device address (no
 *    allocation); make that first call before any stream capture.
 *  - All calls share the one buffer and it keeps the previous call's contents; the
 *    first stage clears what must start at zero.  Calls whose work overlaps on the
 *    GPU (different streams, or different host threads on one device) race on it:
 *    order them on one stream. */
#define FA4D_BWD_NOALLOC_MAX_WORKSPACE ((size_t)64 << 20)
int fa4d_bwd_noalloc(const fa4d_bwd_args* args, void* stream);

/* Block-occupancy pre-pass over a bool mask [Bm, Hm, Tq, Tk] (element strides
 * (batch, head, row), key stride 1; Bm / Hm are the mask's own extents, 1 where it
 * broadcasts).  Writes blocks[((b * Hm + h) * ceil(Tq/128) + qb) * ceil(Tk/128) + kb]
 * = FA4D_BLOCK_EMPTY / _PARTIAL / _FULL for every 128 x 128 block, judged on the
 * in-bounds elements only.  The map is what fa4d_fwd_args.mask_blocks and
 * fa4d_bwd_args.mask_blocks take, and stays valid while the mask is unchanged, so
 * one map serves the forward and backward of every layer sharing the mask.  No
 * counterpart in the reference, whose kernels visit every tile
 * (python/fa2.py:95-124, :242-302). */
enum fa4d_block_state { FA4D_BLOCK_EMPTY = 0, FA4D_BLOCK_PARTIAL = 1, FA4D_BLOCK_FULL = 2 };
size_t fa4d_mask_blocks_size(int32_t Bm, int32_t Hm, int32_t Tq, int32_t Tk);
int fa4d_mask_blocks(const uint8_t* mask, const int64_t mask_stride[3], int32_t Bm, int32_t Hm, int32_t Tq,
                     int32_t Tk, uint8_t* blocks, void* stream);

/* Mask preparation: one pass over a bool mask [Bm, Hm, Tq, Tk] (strides and
 * extents as for fa4d_mask_blocks) that writes into the caller's buffer of
 * fa4d_mask_prepare_size() bytes (256-B aligned):
 *   - the block map of fa4d_mask_blocks (byte offset 0);
 *   - row bits: per (b, h) a [ceil(Tk/128)][Tq][4] array of uint32 whose entry
 *     (kt, q, w) holds the flags of keys 128*kt + 32*w + 0..31 for query q;
 *   - column bits: per (b, h) a [ceil(Tq/64)][Tk][2] array of uint32 whose entry
 *     (qt, k, w) holds the flags of queries 64*qt + 32*w + 0..31 for key k;
 *   - key-tile order: per (b, h) a [ceil(Tk/128)] array of int32 listing the key
 *     tiles by decreasing number of non-EMPTY 128-row query blocks (ties by index;
 *     the identity past 1024 key tiles); the backward launches its key tiles in this
 *     order so the longest CTAs start first;
 * with flags past Tk / Tq zero.  The forward reads one 16-byte row-bit word group
 * per query row and key tile, the backward one 8-byte column-bit group per key and
 * query tile, instead of 128 or 64 mask bytes.  Like the block map, the buffer stays
 * valid while the mask is unchanged (one preparation serves every call sharing the
 * mask).  No counterpart in the reference, which reads the bool mask per element
 * (python/fa2.py:108, :274-280). */
size_t fa4d_mask_prepare_size(int32_t Bm, int32_t Hm, int32_t Tq, int32_t Tk);
int fa4d_mask_prepare(const uint8_t* mask, const int64_t mask_stride[3], int32_t Bm, int32_t Hm, int32_t Tq,
                      int32_t Tk, void* prepared, void* stream);

/* Packed sequences without a mask tensor: per-token document ids doc_q [Bm, Tq] and
 * doc_k [Bm, Tk] (int32, batch strides doc_stride[0] / doc_stride[1] in elements, 0 to
 * broadcast one row over the batch; unit token stride) define keep(q, k) =
 * doc_q[q] == doc_k[k] && doc_q[q] >= 0 (a negative id marks padding, which attends
 * to nothing).  Writes the same prepared-mask buffer as fa4d_mask_prepare with
 * Hm = 1 (fa4d_mask_prepare_size(Bm, 1, Tq, Tk) bytes), reading O(T) ids instead of
 * O(T^2) mask bytes; pass it as mask_prepared with mask == NULL (Bm must be B).
 * In this mode a query row that keeps no key (padding) gets O = 0 and LSE = -inf
 * rather than the NaN a fully masked row gives, so padding adds nothing to dK / dV.
 * The reference's header advertises right-padded / packed support
 * (python/fa2.py:1) but implements it only through a dense 4D mask. */
int fa4d_mask_prepare_docs(const int32_t* doc_q, const int32_t* doc_k, const int64_t doc_stride[2], int32_t Bm,
                           int32_t Tq, int32_t Tk, void* prepared, void* stream);

/* Message for the last non-zero return on this thread ("" if none). */
const char* fa4d_last_error(void);

/* Reads (and with clear != 0 resets) the status word of CUDA device `device`
 * after synchronising `stream`: 0 = no kernel gave up a bounded wait; otherwise a
 * bit set of FA4D_DEV_* flags.  Returns a negative FA4D_ERR_* code if the read
 * fails.  No counterpart in the reference (its kernels have no bounded waits). */
#define FA4D_DEV_TIMEOUT_FWD 1
#define FA4D_DEV_TIMEOUT_BWD 2
#define FA4D_DEV_TIMEOUT_CHECK 4
/* A kernel whose shared-memory layout leaves no alignment slack found its dynamic shared
 * memory base not 1024-byte aligned and returned without computing (not seen on B200). */
#define FA4D_DEV_SMEM_ALIGN 8
int fa4d_device_status(int device, void* stream, int clear);

/* Diagnostic (no counterpart in the reference): runs the kernels' bounded mbarrier
 * wait on a barrier nothing completes, with a limit of `limit_cycles` SM clocks
 * (1..1e9), on the device that is current for the calling thread.  The wait gives up,
 * the kernel sets FA4D_DEV_TIMEOUT_CHECK in the status word and returns; read and
 * clear it with fa4d_device_status.  Exercises the timeout path without any fault. */
int fa4d_check_wait_timeout(int device, int64_t limit_cycles, void* stream);

/* FA4D_ABI_VERSION of the loaded library. */
int fa4d_abi_version(void);

/* Diagnostic (no counterpart in the reference): writes out[i] = e(x_i)/exp2f(x_i) - 1
 * for n points x_i evenly spaced over [lo, hi], where e is the polynomial exp2 the
 * forward kernel evaluates on the FMA pipe for part of its exponentials.  `out` is a
 * device buffer of n floats. */
int fa4d_check_exp2(float* out, int32_t n, float lo, float hi, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FA4D_H_ */
