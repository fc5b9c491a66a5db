// fa4d_api.cu — the C ABI declared in include/fa4d.h: argument validation, TMA
// tensor-map encoding and kernel dispatch.  No allocation happens here; every
// buffer (including the backward workspace) is owned by the caller.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>

#include "fa4d.h"
#include "fa4d_kernels.h"

namespace {

// Device status word: kernels OR FA4D_DEV_* bits into it when a bounded wait gives up.
__device__ int g_status_word = 0;

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

int ok() {
  g_last_error.clear();
  return FA4D_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Address of g_status_word on the current device, looked up once per device.
int* status_word_ptr() {
  static std::mutex mu;
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Makes the device that owns `ptr` current for this library on the calling thread.
// The library links its own CUDA runtime, so the caller's current-device setting
// is not visible here; the driver calls below (tensor-map encoding) need the
// owning device's context current on this thread (autograd runs backward on a
// worker thread of its own).
int bind_device_of(const void* ptr, const char* name) {
  cudaPointerAttributes at;
  cudaError_t e = cudaPointerGetAttributes(&at, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(FA4D_ERR_INVALID, "%s: not a CUDA pointer (%s)", name, cudaGetErrorString(e));
  }
  if (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged)
    return fail(FA4D_ERR_INVALID, "%s: not device memory", name);
  if ((e = cudaSetDevice(at.device)) != cudaSuccess)
    return fail(FA4D_ERR_CUDA, "cudaSetDevice(%d) failed: %s", at.device, cudaGetErrorString(e));
  return FA4D_OK;
}

// Tensor map over a [B, T, H, D] 16-bit tensor given element strides (b, t, h):
// dims (D, T, H, B), box (64, rows, 1, 1), 128-B swizzle, zero fill out of bounds.
int encode_bthd(CUtensorMap* m, const void* ptr, int B, int T, int H, int D, const int64_t st[3], int rows,
                bool bf16, const char* name) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(FA4D_ERR_DRIVER, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  if (!aligned(ptr, 16)) return fail(FA4D_ERR_LAYOUT, "%s: base address is not 16-byte aligned", name);
  const int64_t sz[3] = {B, T, H};
  int64_t bytes[3];
  for (int i = 0; i < 3; ++i) {
    bytes[i] = st[i] * 2;
    // A size-1 dimension is never stepped over; give it a valid stride that is at
    // least as large as the whole tensor so no size rule can trip on it.
    if (sz[i] == 1) bytes[i] = static_cast<int64_t>(D) * 2 * B * T * H;
    if (bytes[i] <= 0 || bytes[i] % 16 != 0 || bytes[i] >= (int64_t(1) << 40))
      return fail(FA4D_ERR_LAYOUT, "%s: stride %lld (elements) is not a positive multiple of 8", name,
                  static_cast<long long>(st[i]));
  }
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(bytes[1]), static_cast<cuuint64_t>(bytes[2]),
                           static_cast<cuuint64_t>(bytes[0])};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FA4D_ERR_DRIVER, "%s: cuTensorMapEncodeTiled failed (%d)", name, int(r));
  return FA4D_OK;
}

// Tensor map over a [B or 1, H or 1, Tq, Tk] mask (1-byte) or score (4-byte) tensor
// given element strides (b, h, row): dims (Tk, Tq, H', B') with a broadcast (stride
// 0) dimension given extent 1, box (128 bytes of keys, `rows` rows, 1, 1), 128-B swizzle,
// zero fill out of bounds.  Returns false when the layout cannot be described by a
// tensor map (unaligned base or strides); the kernels then load from global memory.
bool encode_bias(CUtensorMap* m, const void* ptr, int B, int H, int Tq, int Tk, const int64_t st[3], int esize,
                 int rows = 128) {
  auto enc = tensor_map_encoder();
  if (!enc || !ptr || !aligned(ptr, 16)) return false;
  const int64_t row = st[2] * esize;
  if (row <= 0 || row % 16 != 0 || row >= (int64_t(1) << 40)) return false;
  const int64_t ext_h = st[1] == 0 ? 1 : H, ext_b = st[0] == 0 ? 1 : B;
  int64_t sh = st[1] * esize, sb = st[0] * esize;
  // A size-1 dimension is never stepped over; give it a stride past the whole tensor.
  const int64_t span = row * Tq * ext_h * ext_b;
  if (ext_h == 1) sh = span;
  if (ext_b == 1) sb = span;
  if (sh <= 0 || sh % 16 != 0 || sh >= (int64_t(1) << 40) || sb <= 0 || sb % 16 != 0 || sb >= (int64_t(1) << 40))
    return false;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(Tk), static_cast<cuuint64_t>(Tq), static_cast<cuuint64_t>(ext_h),
                        static_cast<cuuint64_t>(ext_b)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(row), static_cast<cuuint64_t>(sh), static_cast<cuuint64_t>(sb)};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / esize), static_cast<cuuint32_t>(rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, esize == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4,
                   const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int nblocks(int T) { return (T + 127) / 128; }

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Byte offsets inside a prepared-mask buffer: [block map][row bits][column bits]
// [key-tile order], each region starting on a 256-byte boundary.
struct PrepLayout {
  size_t blocks, row_bits, col_bits, kb_order, total;
  int nqb, nkb, nqt;
};
PrepLayout prep_layout(int Bm, int Hm, int Tq, int Tk) {
  PrepLayout L;
  L.nqb = nblocks(Tq);
  L.nkb = nblocks(Tk);
  L.nqt = (Tq + 63) / 64;
  const size_t bh = static_cast<size_t>(Bm) * Hm;
  L.blocks = 0;
  L.row_bits = align256(bh * L.nqb * L.nkb);
  L.col_bits = L.row_bits + align256(bh * L.nkb * static_cast<size_t>(Tq) * 16);
  L.kb_order = L.col_bits + align256(bh * L.nqt * static_cast<size_t>(Tk) * 8);
  L.total = L.kb_order + align256(bh * L.nkb * sizeof(int32_t));
  return L;
}

// Points the kernel parameters at the block map of a prepared mask
// (fa4d_mask_prepare) with extents Bm x Hm; returns its layout for the bit arrays.
template <class P>
PrepLayout use_prepared_map(P& p, const void* prepared, int Bm, int Hm, int Tq, int Tk) {
  const PrepLayout L = prep_layout(Bm, Hm, Tq, Tk);
  p.mask_blocks = static_cast<const uint8_t*>(prepared) + L.blocks;
  p.mb_stride[0] = Bm > 1 ? static_cast<int64_t>(Hm) * L.nqb * L.nkb : 0;
  p.mb_stride[1] = Hm > 1 ? static_cast<int64_t>(L.nqb) * L.nkb : 0;
  return L;
}

// Width the kernels compute at for head dim D.  D = 96 runs the D = 128 kernels: the
// tensor maps (extent 96) zero-fill columns 96..127 of every Q, K, V and dO tile, so
// those columns of S contribute nothing and those of O, dQ, dK, dV come out zero; the
// kernels store only the first 96.  Accumulator workspaces use the compute width.
int compute_dim(int D) { return D == 96 ? 128 : D; }

int check_common(int B, int Tq, int Tk, int Hq, int Hk, int D, int dtype, int causal, float scale) {
  if (B < 1 || Tq < 1 || Tk < 1 || Hq < 1 || Hk < 1)
    return fail(FA4D_ERR_INVALID, "sizes must be positive (B=%d Tq=%d Tk=%d Hq=%d Hk=%d)", B, Tq, Tk, Hq, Hk);
  if (Hq % Hk != 0)
    return fail(FA4D_ERR_INVALID, "query heads (%d) must be divisible by key/value heads (%d)", Hq, Hk);
  if (B > 65535 || Hq > 65535) return fail(FA4D_ERR_INVALID, "B and Hq must be <= 65535");
  if ((Tq + 255) / 256 > 65535 || (Tk + 127) / 128 > 65535)
    return fail(FA4D_ERR_UNSUPPORTED, "sequence too long for the launch grid (Tq <= 16M, Tk <= 8M)");
  if (Tq > (1 << 30) || Tk > (1 << 30)) return fail(FA4D_ERR_INVALID, "sequence length too large");
  if (D != 64 && D != 96 && D != 128 && D != 256)
    return fail(FA4D_ERR_UNSUPPORTED, "head dim %d is not built (64, 96, 128, 256)", D);
  if (dtype != FA4D_BF16 && dtype != FA4D_F16) return fail(FA4D_ERR_INVALID, "dtype %d is not bf16/f16", dtype);
  if (causal < FA4D_CAUSAL_NONE || causal > FA4D_CAUSAL_BOTTOM_RIGHT)
    return fail(FA4D_ERR_INVALID, "causal mode %d is unknown", causal);
  if (!(scale == scale)) return fail(FA4D_ERR_INVALID, "scale is NaN");
  return FA4D_OK;
}

// Row pointers of a [.., D] output written with 16-byte stores.
int check_rows16(const void* ptr, const int64_t st[3], const char* name) {
  if (!ptr) return fail(FA4D_ERR_INVALID, "%s is NULL", name);
  if (!aligned(ptr, 16)) return fail(FA4D_ERR_LAYOUT, "%s: base address is not 16-byte aligned", name);
  for (int i = 0; i < 3; ++i)
    if (st[i] % 8 != 0) return fail(FA4D_ERR_LAYOUT, "%s: strides must be multiples of 8 elements", name);
  return FA4D_OK;
}

int causal_offset(int causal, int Tq, int Tk) { return causal == FA4D_CAUSAL_BOTTOM_RIGHT ? Tk - Tq : 0; }

int64_t lse_ld_of(int Tq) { return (static_cast<int64_t>(Tq) + 127) / 128 * 128; }

// Bytes of one set of split-group partial slices [S][B, Tk, Hk, D] fp32.
size_t part_bytes(int S, int B, int Tk, int Hk, int D) {
  return (static_cast<size_t>(S) * B * Tk * Hk * D * sizeof(float) + 255) / 256 * 256;
}

int sm_count();

// Bytes of the fp32 dQ accumulator [B, Hq, lse_ld, Dc] at the head of the backward
// workspace, rounded to 256; none at D = 256, where dQ always comes from the ordered
// pass (plan_bwd), which writes dQ directly.
size_t dq_acc_bytes(int B, int Tq, int Hq, int D) {
  if (D == 256) return 0;
  const size_t dq = static_cast<size_t>(B) * Hq * lse_ld_of(Tq) * compute_dim(D) * sizeof(float);
  return (dq + 255) / 256 * 256;
}

// Group split of the backward: the query-head group of each (key tile, KV head, batch)
// is split over S CTAs (a power of two dividing the group size, at most 8) when that
// shortens the estimated run.  A CTA takes G / S heads x its key tile's query tiles
// (about 1.5 us per 64-row tile at D = 128, 0.9 us at D = 64) plus about 5 us of fixed
// cost; a split adds the fp32 partial slices of dK and dV (written, then summed by
// dkv_convert_kernel) at about 6 TB/s.  When every key tile has about the same number of
// query tiles (no causal limit, or a band as in bottom-right alignment with Tq < Tk),
// the grid runs in ceil(CTAs / SMs) equal waves, so splitting also fills a last wave
// that would run mostly empty (512 CTAs on 148 SMs: 3.46 waves, the fourth under half
// full).  Otherwise the longest-first grid order balances the SMs and the estimate is
// the larger of the total work per SM and the longest CTA, so only grids too small for
// the GPU (MQA, short key sequences) are split.
// Query tiles (64 rows) per 128-key tile of the backward: mean and maximum over the
// key tiles, and whether they are about equal (every key tile within 1.2 x the mean).
struct KeyTileWork {
  double mean_nq, max_nq;
  bool equal;
};
KeyTileWork key_tile_work(int Tq, int Tk, int causal) {
  const int nkb = (Tk + 127) / 128;
  const int nqt = (Tq + 63) / 64;
  KeyTileWork w{static_cast<double>(nqt), static_cast<double>(nqt), true};
  if (causal) {
    const long long off = causal_offset(causal, Tq, Tk);
    double sum = 0.0;
    w.max_nq = 0.0;
    for (int kb = 0; kb < nkb; ++kb) {
      const long long qmin = 128LL * kb - off;
      const int first = qmin <= 0 ? 0 : static_cast<int>(qmin / 64);
      const double n = first < nqt ? nqt - first : 0;
      sum += n;
      w.max_nq = n > w.max_nq ? n : w.max_nq;
    }
    w.mean_nq = sum / nkb;
  }
  w.equal = w.max_nq <= 1.2 * w.mean_nq;
  return w;
}

int group_split(int B, int Tq, int Tk, int Hq, int Hk, int D, int causal) {
  const int G = Hq / Hk;
  const int nkb = (Tk + 127) / 128;
  // At D = 256 a cluster of two CTAs shares each key tile (one per half of the products).
  const double base = static_cast<double>(nkb) * Hk * B * (D == 256 ? 2 : 1);
  const double sms = sm_count();
  const double tile_us = D == 256 ? 2.0 : (D > 64 ? 1.5 : 0.9);
  const KeyTileWork w = key_tile_work(Tq, Tk, causal);
  const double mean_nq = w.mean_nq, max_nq = w.max_nq;
  const bool uniform = w.equal;
  const double kv_elems = static_cast<double>(B) * Tk * Hk * D;
  double best = 0.0;
  int best_s = 1;
  for (int S = 1; S <= 8 && G % S == 0 && static_cast<int64_t>(Hk) * S <= 65535; S *= 2) {
    const double per_head = static_cast<double>(G) / S * tile_us;
    double t = uniform ? std::ceil(base * S / sms) * (per_head * mean_nq + 5.0)
                       : std::max(base * S / sms * (per_head * mean_nq + 5.0), per_head * max_nq + 5.0);
    if (S > 1) t += kv_elems * 2.0 * (8.0 * S + 2.0) / 6.0e6;
    if (S == 1 || t < 0.98 * best) {
      best = t;
      best_s = S;
    }
  }
  return best_s;
}

// SM count of the current device (cached per device).
int sm_count() {
  static std::mutex mu;
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (!counts[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

}  // namespace

extern "C" {

int64_t fa4d_lse_row_stride(int32_t Tq) { return lse_ld_of(Tq); }

size_t fa4d_bwd_workspace_size(int32_t B, int32_t Tq, int32_t Hq, int32_t D) {
  const size_t dq_al = dq_acc_bytes(B, Tq, Hq, D);
  const size_t delta = static_cast<size_t>(B) * Hq * lse_ld_of(Tq) * sizeof(float);
  return dq_al + (delta + 255) / 256 * 256;
}

int32_t fa4d_bwd_group_split(int32_t B, int32_t Tq, int32_t Tk, int32_t Hq, int32_t Hk, int32_t D, int32_t causal) {
  if (B <= 0 || Tq <= 0 || Tk <= 0 || Hq <= 0 || Hk <= 0 || Hq % Hk != 0) return 0;
  if (causal < FA4D_CAUSAL_NONE || causal > FA4D_CAUSAL_BOTTOM_RIGHT) return 0;
  return group_split(B, Tq, Tk, Hq, Hk, D, causal);
}

size_t fa4d_bwd_workspace_size_ex(int32_t B, int32_t Tq, int32_t Tk, int32_t Hq, int32_t Hk, int32_t D) {
  // The causal mode is not an argument here: size for the largest split any mode picks.
  int S = 1;
  if (B > 0 && Tq > 0 && Tk > 0 && Hq > 0 && Hk > 0 && Hq % Hk == 0)
    for (int c = FA4D_CAUSAL_NONE; c <= FA4D_CAUSAL_BOTTOM_RIGHT; ++c) S = std::max(S, group_split(B, Tq, Tk, Hq, Hk, D, c));
  return fa4d_bwd_workspace_size(B, Tq, Hq, D) + (S > 1 ? 2 * part_bytes(S, B, Tk, Hk, compute_dim(D)) : 0);
}

const char* fa4d_last_error(void) { return g_last_error.c_str(); }

int fa4d_abi_version(void) { return FA4D_ABI_VERSION; }

size_t fa4d_mask_prepare_size(int32_t Bm, int32_t Hm, int32_t Tq, int32_t Tk) {
  if (Bm < 1 || Hm < 1 || Tq < 1 || Tk < 1) return 0;
  return prep_layout(Bm, Hm, Tq, Tk).total;
}

int fa4d_mask_prepare(const uint8_t* mask, const int64_t mask_stride[3], int32_t Bm, int32_t Hm, int32_t Tq,
                      int32_t Tk, void* prepared, void* stream) {
  if (!mask || !mask_stride || !prepared) return fail(FA4D_ERR_INVALID, "mask, mask_stride and prepared are required");
  if (Bm < 1 || Hm < 1 || Tq < 1 || Tk < 1)
    return fail(FA4D_ERR_INVALID, "sizes must be positive (Bm=%d Hm=%d Tq=%d Tk=%d)", Bm, Hm, Tq, Tk);
  if (static_cast<int64_t>(Bm) * Hm > 65535 || nblocks(Tq) > 65535)
    return fail(FA4D_ERR_UNSUPPORTED, "Bm*Hm and ceil(Tq/128) must be <= 65535");
  if (mask_stride[0] < 0 || mask_stride[1] < 0 || mask_stride[2] < 0)
    return fail(FA4D_ERR_INVALID, "mask strides must be non-negative");
  if (!aligned(prepared, 256)) return fail(FA4D_ERR_LAYOUT, "prepared buffer must be 256-byte aligned");
  int rc = bind_device_of(mask, "mask");
  if (rc) return rc;
  const PrepLayout L = prep_layout(Bm, Hm, Tq, Tk);
  fa4d::MaskPrepParams p;
  memset(&p, 0, sizeof(p));
  p.mask = mask;
  for (int i = 0; i < 3; ++i) p.stride[i] = mask_stride[i];
  p.Bm = Bm;
  p.Hm = Hm;
  p.Tq = Tq;
  p.Tk = Tk;
  p.nqb = L.nqb;
  p.nkb = L.nkb;
  p.nqt = L.nqt;
  p.vec = aligned(mask, 16) && Tk % 16 == 0 && mask_stride[0] % 16 == 0 && mask_stride[1] % 16 == 0 &&
          mask_stride[2] % 16 == 0;
  char* base = static_cast<char*>(prepared);
  p.blocks = reinterpret_cast<uint8_t*>(base + L.blocks);
  p.row_bits = reinterpret_cast<uint32_t*>(base + L.row_bits);
  p.col_bits = reinterpret_cast<uint32_t*>(base + L.col_bits);
  p.kb_order = reinterpret_cast<int32_t*>(base + L.kb_order);
  cudaError_t e = fa4d::launch_mask_prepare(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(FA4D_ERR_CUDA, "mask prepare launch failed: %s", cudaGetErrorString(e));
  return ok();
}

int fa4d_mask_prepare_docs(const int32_t* doc_q, const int32_t* doc_k, const int64_t doc_stride[2], int32_t Bm,
                           int32_t Tq, int32_t Tk, void* prepared, void* stream) {
  if (!doc_q || !doc_k || !doc_stride || !prepared)
    return fail(FA4D_ERR_INVALID, "doc_q, doc_k, doc_stride and prepared are required");
  if (Bm < 1 || Tq < 1 || Tk < 1) return fail(FA4D_ERR_INVALID, "sizes must be positive (Bm=%d Tq=%d Tk=%d)", Bm, Tq, Tk);
  if (Bm > 65535 || nblocks(Tq) > 65535) return fail(FA4D_ERR_UNSUPPORTED, "Bm and ceil(Tq/128) must be <= 65535");
  if (doc_stride[0] < 0 || doc_stride[1] < 0) return fail(FA4D_ERR_INVALID, "doc strides must be non-negative");
  if (!aligned(prepared, 256)) return fail(FA4D_ERR_LAYOUT, "prepared buffer must be 256-byte aligned");
  int rc = bind_device_of(doc_q, "doc_q");
  if (rc) return rc;
  const PrepLayout L = prep_layout(Bm, 1, Tq, Tk);
  fa4d::MaskPrepParams p;
  memset(&p, 0, sizeof(p));
  p.Bm = Bm;
  p.Hm = 1;
  p.Tq = Tq;
  p.Tk = Tk;
  p.nqb = L.nqb;
  p.nkb = L.nkb;
  p.nqt = L.nqt;
  p.doc_q = doc_q;
  p.doc_k = doc_k;
  p.doc_q_stride = doc_stride[0];
  p.doc_k_stride = doc_stride[1];
  char* base = static_cast<char*>(prepared);
  p.blocks = reinterpret_cast<uint8_t*>(base + L.blocks);
  p.row_bits = reinterpret_cast<uint32_t*>(base + L.row_bits);
  p.col_bits = reinterpret_cast<uint32_t*>(base + L.col_bits);
  p.kb_order = reinterpret_cast<int32_t*>(base + L.kb_order);
  cudaError_t e = fa4d::launch_mask_prepare(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(FA4D_ERR_CUDA, "document mask prepare launch failed: %s", cudaGetErrorString(e));
  return ok();
}

size_t fa4d_mask_blocks_size(int32_t Bm, int32_t Hm, int32_t Tq, int32_t Tk) {
  if (Bm < 1 || Hm < 1 || Tq < 1 || Tk < 1) return 0;
  return static_cast<size_t>(Bm) * Hm * nblocks(Tq) * nblocks(Tk);
}

int fa4d_mask_blocks(const uint8_t* mask, const int64_t mask_stride[3], int32_t Bm, int32_t Hm, int32_t Tq,
                     int32_t Tk, uint8_t* blocks, void* stream) {
  if (!mask || !mask_stride || !blocks) return fail(FA4D_ERR_INVALID, "mask, mask_stride and blocks are required");
  if (Bm < 1 || Hm < 1 || Tq < 1 || Tk < 1)
    return fail(FA4D_ERR_INVALID, "sizes must be positive (Bm=%d Hm=%d Tq=%d Tk=%d)", Bm, Hm, Tq, Tk);
  if (static_cast<int64_t>(Bm) * Hm > 65535 || nblocks(Tq) > 65535)
    return fail(FA4D_ERR_UNSUPPORTED, "Bm*Hm and ceil(Tq/128) must be <= 65535");
  if (mask_stride[0] < 0 || mask_stride[1] < 0 || mask_stride[2] < 0)
    return fail(FA4D_ERR_INVALID, "mask strides must be non-negative");
  int rc = bind_device_of(mask, "mask");
  if (rc) return rc;
  fa4d::MaskBlocksParams p;
  memset(&p, 0, sizeof(p));
  p.mask = mask;
  for (int i = 0; i < 3; ++i) p.stride[i] = mask_stride[i];
  p.Bm = Bm;
  p.Hm = Hm;
  p.Tq = Tq;
  p.Tk = Tk;
  p.nqb = nblocks(Tq);
  p.nkb = nblocks(Tk);
  p.vec = aligned(mask, 16) && Tk % 16 == 0 && mask_stride[0] % 16 == 0 && mask_stride[1] % 16 == 0 &&
          mask_stride[2] % 16 == 0;
  p.blocks = blocks;
  cudaError_t e = fa4d::launch_mask_blocks(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(FA4D_ERR_CUDA, "mask block pass launch failed: %s", cudaGetErrorString(e));
  return ok();
}

int fa4d_check_exp2(float* out, int32_t n, float lo, float hi, void* stream) {
  if (!out || n < 2) return fail(FA4D_ERR_INVALID, "out must be a device buffer of n >= 2 floats");
  int rc = bind_device_of(out, "out");
  if (rc) return rc;
  cudaError_t e = fa4d::launch_exp2_check(out, n, lo, hi, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(FA4D_ERR_CUDA, "exp2 check launch failed: %s", cudaGetErrorString(e));
  return ok();
}

int fa4d_check_wait_timeout(int device, int64_t limit_cycles, void* stream) {
  if (limit_cycles < 1 || limit_cycles > 1000000000LL)
    return fail(FA4D_ERR_INVALID, "limit_cycles must be in [1, 1e9]");
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail(FA4D_ERR_CUDA, "cudaSetDevice(%d) failed: %s", device, cudaGetErrorString(e));
  int* word = status_word_ptr();
  if (!word) return fail(FA4D_ERR_CUDA, "cannot locate the device status word");
  e = fa4d::launch_wait_timeout_check(word, limit_cycles, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(FA4D_ERR_CUDA, "wait check launch failed: %s", cudaGetErrorString(e));
  return ok();
}

int fa4d_device_status(int device, void* stream, int clear) {
  cudaError_t se = cudaSetDevice(device);
  if (se != cudaSuccess) return fail(FA4D_ERR_CUDA, "cudaSetDevice(%d) failed: %s", device, cudaGetErrorString(se));
  int* word = status_word_ptr();
  if (!word) return fail(FA4D_ERR_CUDA, "cannot locate the device status word");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, word, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && clear) {
    e = cudaMemsetAsync(word, 0, sizeof(int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  }
  if (e != cudaSuccess) return fail(FA4D_ERR_CUDA, "device status read failed: %s", cudaGetErrorString(e));
  return v;
}

int fa4d_fwd(const fa4d_fwd_args* a, void* stream) {
  if (!a) return fail(FA4D_ERR_INVALID, "args is NULL");
  int rc = check_common(a->B, a->Tq, a->Tk, a->Hq, a->Hk, a->D, a->dtype, a->causal, a->scale);
  if (rc) return rc;
  if (!a->q || !a->k || !a->v || !a->o || !a->lse) return fail(FA4D_ERR_INVALID, "q, k, v, o and lse are required");
  if ((rc = check_rows16(a->o, a->o_stride, "o"))) return rc;
  if ((rc = bind_device_of(a->q, "q"))) return rc;
  const bool bf16 = a->dtype == FA4D_BF16;
  fa4d::FwdParams p;
  memset(&p, 0, sizeof(p));
  if ((rc = encode_bthd(&p.tm_q, a->q, a->B, a->Tq, a->Hq, a->D, a->q_stride, 128, bf16, "q"))) return rc;
  if ((rc = encode_bthd(&p.tm_k, a->k, a->B, a->Tk, a->Hk, a->D, a->k_stride, 128, bf16, "k"))) return rc;
  if ((rc = encode_bthd(&p.tm_v, a->v, a->B, a->Tk, a->Hk, a->D, a->v_stride, 128, bf16, "v"))) return rc;
  p.o = a->o;
  p.lse = a->lse;
  p.mask = a->mask;
  p.score = a->score;
  for (int i = 0; i < 3; ++i) {
    p.o_stride[i] = a->o_stride[i];
    p.mask_stride[i] = a->mask_stride[i];
    p.score_stride[i] = a->score_stride[i];
  }
  p.B = a->B;
  p.Tq = a->Tq;
  p.Tk = a->Tk;
  p.Hq = a->Hq;
  p.Hk = a->Hk;
  p.lse_ld = static_cast<int32_t>(lse_ld_of(a->Tq));
  p.causal = a->causal != FA4D_CAUSAL_NONE;
  p.causal_off = causal_offset(a->causal, a->Tq, a->Tk);
  p.scale_log2 = static_cast<float>(static_cast<double>(a->scale) * 1.4426950408889634);
  p.mask_vec = a->mask && aligned(a->mask, 4) && a->mask_stride[0] % 4 == 0 && a->mask_stride[1] % 4 == 0 &&
               a->mask_stride[2] % 4 == 0;
  p.score_vec = a->score && aligned(a->score, 16) && a->score_stride[0] % 4 == 0 && a->score_stride[1] % 4 == 0 &&
                a->score_stride[2] % 4 == 0;
  p.status = status_word_ptr();
  if (!p.status) return fail(FA4D_ERR_CUDA, "cannot locate the device status word");
  p.nkb = nblocks(a->Tk);
  if (a->mask_prepared) {
    if (!aligned(a->mask_prepared, 256)) return fail(FA4D_ERR_LAYOUT, "mask_prepared must be 256-byte aligned");
    // Without a mask pointer the buffer came from fa4d_mask_prepare_docs: Bm = B, Hm = 1.
    const int Bm = (!a->mask || a->mask_stride[0]) ? a->B : 1, Hm = (a->mask && a->mask_stride[1]) ? a->Hq : 1;
    const PrepLayout L = use_prepared_map(p, a->mask_prepared, Bm, Hm, a->Tq, a->Tk);
    p.mask_bits = reinterpret_cast<const uint32_t*>(static_cast<const char*>(a->mask_prepared) + L.row_bits);
    p.empty_rows_zero = a->mask == nullptr;
    const int64_t per_head = static_cast<int64_t>(L.nkb) * a->Tq * 4;
    p.mbits_stride[0] = Bm > 1 ? per_head * Hm : 0;
    p.mbits_stride[1] = Hm > 1 ? per_head : 0;
  } else if (a->mask && a->mask_blocks) {
    p.mask_blocks = a->mask_blocks;
    p.mb_stride[0] = a->mask_blocks_stride[0];
    p.mb_stride[1] = a->mask_blocks_stride[1];
  }
  if (a->score) {
    p.bias_tma = encode_bias(&p.tm_score, a->score, a->B, a->Hq, a->Tq, a->Tk, a->score_stride, 4);
  }
  p.d_out = a->D;
  cudaError_t e = fa4d::launch_fwd(p, compute_dim(a->D), bf16, a->mask != nullptr || a->mask_prepared != nullptr,
                                   a->score != nullptr, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(FA4D_ERR_CUDA, "forward launch failed: %s", cudaGetErrorString(e));
  return ok();
}

}  // extern "C"

namespace {

struct BwdPlan {
  fa4d::BwdParams main;
  fa4d::DqParams dq;  // deterministic mode only
  bool deterministic;
  fa4d::PrepParams prep;
  fa4d::ConvertParams convert;
  fa4d::DkvConvertParams dkv;
  bool bf16;
  int D;
  bool has_mask, has_score;
};

// Validates a backward call and fills the parameter blocks of its three stages.
int plan_bwd(const fa4d_bwd_args* a, BwdPlan* plan) {
  if (!a) return fail(FA4D_ERR_INVALID, "args is NULL");
  int rc = check_common(a->B, a->Tq, a->Tk, a->Hq, a->Hk, a->D, a->dtype, a->causal, a->scale);
  if (rc) return rc;
  if (!a->q || !a->k || !a->v || !a->o || !a->dout || !a->lse)
    return fail(FA4D_ERR_INVALID, "q, k, v, o, dout and lse are required");
  if (a->deterministic != 0 && a->deterministic != 1) return fail(FA4D_ERR_INVALID, "deterministic must be 0 or 1");
  if (a->D == 256 && (rc = check_rows16(a->v, a->v_stride, "v"))) return rc;
  if ((rc = check_rows16(a->dq, a->dq_stride, "dq"))) return rc;
  if ((rc = check_rows16(a->dk, a->dk_stride, "dk"))) return rc;
  if ((rc = check_rows16(a->dv, a->dv_stride, "dv"))) return rc;
  if ((rc = check_rows16(a->o, a->o_stride, "o"))) return rc;
  if ((rc = check_rows16(a->dout, a->do_stride, "dout"))) return rc;
  const size_t need = fa4d_bwd_workspace_size(a->B, a->Tq, a->Hq, a->D);
  if (!a->workspace || a->workspace_bytes < need || !aligned(a->workspace, 256))
    return fail(FA4D_ERR_WORKSPACE, "workspace must be 256-B aligned and hold %zu bytes (got %zu)", need,
                a->workspace_bytes);
  if ((rc = bind_device_of(a->q, "q"))) return rc;
  const bool bf16 = a->dtype == FA4D_BF16;
  const int64_t lse_ld = lse_ld_of(a->Tq);
  float* dq_acc = a->D == 256 ? nullptr : static_cast<float*>(a->workspace);  // see dq_acc_bytes
  const int Dc = compute_dim(a->D);
  float* delta = reinterpret_cast<float*>(static_cast<char*>(a->workspace) + dq_acc_bytes(a->B, a->Tq, a->Hq, a->D));
  int* status = status_word_ptr();
  if (!status) return fail(FA4D_ERR_CUDA, "cannot locate the device status word");

  memset(plan, 0, sizeof(*plan));
  plan->bf16 = bf16;
  plan->D = Dc;
  plan->has_mask = a->mask != nullptr || a->mask_prepared != nullptr;
  plan->has_score = a->score != nullptr;
  fa4d::BwdParams& p = plan->main;
  if ((rc = encode_bthd(&p.tm_q, a->q, a->B, a->Tq, a->Hq, a->D, a->q_stride, 64, bf16, "q"))) return rc;
  if ((rc = encode_bthd(&p.tm_do, a->dout, a->B, a->Tq, a->Hq, a->D, a->do_stride, 64, bf16, "dout"))) return rc;
  if ((rc = encode_bthd(&p.tm_k, a->k, a->B, a->Tk, a->Hk, a->D, a->k_stride, 128, bf16, "k"))) return rc;
  if ((rc = encode_bthd(&p.tm_v, a->v, a->B, a->Tk, a->Hk, a->D, a->v_stride, 128, bf16, "v"))) return rc;
  p.lse = a->lse;
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.d_out = a->D;
  p.dk = a->dk;
  p.dv = a->dv;
  p.v = a->v;
  p.k = a->k;
  p.mask = a->mask;
  p.score = a->score;
  for (int i = 0; i < 3; ++i) {
    p.dk_stride[i] = a->dk_stride[i];
    p.dv_stride[i] = a->dv_stride[i];
    p.v_stride[i] = a->v_stride[i];
    p.k_stride[i] = a->k_stride[i];
    p.mask_stride[i] = a->mask_stride[i];
    p.score_stride[i] = a->score_stride[i];
  }
  p.B = a->B;
  p.Tq = a->Tq;
  p.Tk = a->Tk;
  p.Hq = a->Hq;
  p.Hk = a->Hk;
  p.lse_ld = static_cast<int32_t>(lse_ld);
  p.causal = a->causal != FA4D_CAUSAL_NONE;
  p.causal_off = causal_offset(a->causal, a->Tq, a->Tk);
  p.scale_log2 = static_cast<float>(static_cast<double>(a->scale) * 1.4426950408889634);
  p.scale = a->scale;
  p.status = status;
  p.nkb = nblocks(a->Tk);
  if (a->mask_prepared) {
    if (!aligned(a->mask_prepared, 256)) return fail(FA4D_ERR_LAYOUT, "mask_prepared must be 256-byte aligned");
    const int Bm = (!a->mask || a->mask_stride[0]) ? a->B : 1, Hm = (a->mask && a->mask_stride[1]) ? a->Hq : 1;
    const PrepLayout L = use_prepared_map(p, a->mask_prepared, Bm, Hm, a->Tq, a->Tk);
    p.mask_bits_t = reinterpret_cast<const uint32_t*>(static_cast<const char*>(a->mask_prepared) + L.col_bits);
    const int64_t per_head = static_cast<int64_t>(L.nqt) * a->Tk * 2;
    p.mbt_stride[0] = Bm > 1 ? per_head * Hm : 0;
    p.mbt_stride[1] = Hm > 1 ? per_head : 0;
    // Key tiles in the prepared order, longest first (D = 256 runs its own grid).
    if (compute_dim(a->D) != 256 && static_cast<int64_t>(L.nkb) * a->B <= 65535) {
      p.kb_order = reinterpret_cast<const int32_t*>(static_cast<const char*>(a->mask_prepared) + L.kb_order);
      p.ko_stride[0] = Bm > 1 ? static_cast<int64_t>(Hm) * L.nkb : 0;
      p.ko_stride[1] = Hm > 1 ? L.nkb : 0;
    }
  } else if (a->mask && a->mask_blocks) {
    p.mask_blocks = a->mask_blocks;
    p.mb_stride[0] = a->mask_blocks_stride[0];
    p.mb_stride[1] = a->mask_blocks_stride[1];
  }
  if (a->score) p.score_pf = encode_bias(&p.tm_score, a->score, a->B, a->Hq, a->Tq, a->Tk, a->score_stride, 4, 64);
  // Group split (see group_split), used when the caller's workspace was sized with
  // fa4d_bwd_workspace_size_ex; otherwise one CTA per key tile takes the whole group.
  // Equal-work grids without a block map run key tiles fastest (see BwdParams).
  p.kb_fastest = (!p.mask_blocks && key_tile_work(a->Tq, a->Tk, a->causal).equal) ? 1 : 0;
  p.g_split = 1;
  {
    const int S = group_split(a->B, a->Tq, a->Tk, a->Hq, a->Hk, a->D, a->causal);
    const size_t base_ws = fa4d_bwd_workspace_size(a->B, a->Tq, a->Hq, a->D);
    const size_t pb = part_bytes(S, a->B, a->Tk, a->Hk, Dc);
    if (S > 1 && a->workspace_bytes >= base_ws + 2 * pb) {
      {
        p.g_split = S;
        p.part_stride = static_cast<int64_t>(a->B) * a->Tk * a->Hk * Dc;
        p.dk_part = reinterpret_cast<float*>(static_cast<char*>(a->workspace) + base_ws);
        p.dv_part = reinterpret_cast<float*>(static_cast<char*>(a->workspace) + base_ws + pb);
        fa4d::DkvConvertParams& kp = plan->dkv;
        kp.dk_part = p.dk_part;
        kp.dv_part = p.dv_part;
        kp.part_stride = p.part_stride;
        kp.n_split = S;
        kp.dk = a->dk;
        kp.dv = a->dv;
        for (int i = 0; i < 3; ++i) {
          kp.dk_stride[i] = a->dk_stride[i];
          kp.dv_stride[i] = a->dv_stride[i];
        }
        kp.B = a->B;
        kp.Tk = a->Tk;
        kp.Hk = a->Hk;
        kp.D = Dc;
        kp.d_out = a->D;
      }
    }
  }

  // At D = 256 dQ always comes from the ordered pass: the D = 256 main kernel has no
  // dQ products (measured slower there than the separate pass).
  if (a->deterministic || a->D == 256) {
    // dQ from its own kernel (one CTA per query tile, key tiles in order); the main
    // kernel skips its dQ products and nothing is accumulated.
    plan->deterministic = true;
    p.skip_dq = 1;
    fa4d::DqParams& d = plan->dq;
    if ((rc = encode_bthd(&d.tm_q, a->q, a->B, a->Tq, a->Hq, a->D, a->q_stride, 128, bf16, "q"))) return rc;
    if ((rc = encode_bthd(&d.tm_do, a->dout, a->B, a->Tq, a->Hq, a->D, a->do_stride, 128, bf16, "dout"))) return rc;
    // Key tiles are loaded whole, or in 64-row halves at D = 256 (fa4d_dq256.cu).
    const int kv_rows = a->D == 256 ? 64 : 128;
    if ((rc = encode_bthd(&d.tm_k, a->k, a->B, a->Tk, a->Hk, a->D, a->k_stride, kv_rows, bf16, "k"))) return rc;
    if ((rc = encode_bthd(&d.tm_v, a->v, a->B, a->Tk, a->Hk, a->D, a->v_stride, kv_rows, bf16, "v"))) return rc;
    d.lse = a->lse;
    d.delta = delta;
    d.dq = a->dq;
    d.d_out = a->D;
    d.mask = a->mask;
    d.score = a->score;
    for (int i = 0; i < 3; ++i) {
      d.dq_stride[i] = a->dq_stride[i];
      d.mask_stride[i] = a->mask_stride[i];
      d.score_stride[i] = a->score_stride[i];
    }
    d.mask_blocks = p.mask_blocks;
    d.mb_stride[0] = p.mb_stride[0];
    d.mb_stride[1] = p.mb_stride[1];
    d.nkb = p.nkb;
    if (a->mask_prepared) {
      const int Bm = (!a->mask || a->mask_stride[0]) ? a->B : 1, Hm = (a->mask && a->mask_stride[1]) ? a->Hq : 1;
      const PrepLayout L = prep_layout(Bm, Hm, a->Tq, a->Tk);
      d.mask_bits = reinterpret_cast<const uint32_t*>(static_cast<const char*>(a->mask_prepared) + L.row_bits);
      const int64_t per_head = static_cast<int64_t>(L.nkb) * a->Tq * 4;
      d.mbits_stride[0] = Bm > 1 ? per_head * Hm : 0;
      d.mbits_stride[1] = Hm > 1 ? per_head : 0;
    }
    d.mask_vec = a->mask && aligned(a->mask, 4) && a->mask_stride[0] % 4 == 0 && a->mask_stride[1] % 4 == 0 &&
                 a->mask_stride[2] % 4 == 0;
    d.score_vec = a->score && aligned(a->score, 16) && a->score_stride[0] % 4 == 0 &&
                  a->score_stride[1] % 4 == 0 && a->score_stride[2] % 4 == 0;
    d.B = a->B;
    d.Tq = a->Tq;
    d.Tk = a->Tk;
    d.Hq = a->Hq;
    d.Hk = a->Hk;
    d.lse_ld = static_cast<int32_t>(lse_ld);
    d.causal = p.causal;
    d.causal_off = p.causal_off;
    d.scale_log2 = p.scale_log2;
    d.scale = a->scale;
    d.status = status;
  }

  fa4d::PrepParams& pp = plan->prep;
  pp.o = a->o;
  pp.dout = a->dout;
  pp.delta = delta;
  pp.dq_acc = plan->deterministic ? nullptr : dq_acc;
  for (int i = 0; i < 3; ++i) {
    pp.o_stride[i] = a->o_stride[i];
    pp.do_stride[i] = a->do_stride[i];
  }
  pp.B = a->B;
  pp.Tq = a->Tq;
  pp.Hq = a->Hq;
  pp.D = Dc;
  pp.d_out = a->D;
  pp.lse_ld = static_cast<int32_t>(lse_ld);

  fa4d::ConvertParams& cp = plan->convert;
  cp.dq_acc = dq_acc;
  cp.dq = a->dq;
  for (int i = 0; i < 3; ++i) cp.dq_stride[i] = a->dq_stride[i];
  cp.B = a->B;
  cp.Tq = a->Tq;
  cp.Hq = a->Hq;
  cp.D = Dc;
  cp.d_out = a->D;
  cp.lse_ld = static_cast<int32_t>(lse_ld);
  cp.scale = a->scale;
  return FA4D_OK;
}

int run_stage(const BwdPlan& plan, int stage, cudaStream_t s) {
  cudaError_t e = cudaSuccess;
  const char* what = "";
  if (stage == 0) {
    e = fa4d::launch_bwd_prep(plan.prep, plan.bf16, s);
    what = "backward preprocess";

  } else if (stage == 1) {
    e = fa4d::launch_bwd(plan.main, plan.D, plan.bf16, plan.has_mask, plan.has_score, s);
    what = "backward main";
  } else {
    if (plan.deterministic) {
      e = fa4d::launch_dq(plan.dq, plan.D, plan.bf16, plan.has_mask, plan.has_score, s);
      what = "deterministic dQ";
    } else {
      e = fa4d::launch_dq_convert(plan.convert, plan.bf16, s);
      what = "dQ convert";
    }
    if (e == cudaSuccess && plan.main.g_split > 1) e = fa4d::launch_dkv_convert(plan.dkv, plan.bf16, s);
  }
  if (e != cudaSuccess) return fail(FA4D_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return FA4D_OK;
}

int bwd_stages(const fa4d_bwd_args* a, int first, int last, void* stream) {
  BwdPlan plan;
  int rc = plan_bwd(a, &plan);
  if (rc) return rc;
  for (int st = first; st <= last; ++st)
    if ((rc = run_stage(plan, st, static_cast<cudaStream_t>(stream)))) return rc;
  return ok();
}

}  // namespace

extern "C" {

int fa4d_bwd(const fa4d_bwd_args* a, void* stream) { return bwd_stages(a, 0, 2, stream); }
int fa4d_bwd_preprocess(const fa4d_bwd_args* a, void* stream) { return bwd_stages(a, 0, 0, stream); }
int fa4d_bwd_main(const fa4d_bwd_args* a, void* stream) { return bwd_stages(a, 1, 1, stream); }
int fa4d_bwd_dq_convert(const fa4d_bwd_args* a, void* stream) { return bwd_stages(a, 2, 2, stream); }

}  // extern "C"


// ---------------------------------------------------------------------------------
// Backward without any allocation by anyone.
//
// Some callers cannot hand the library a workspace: hosts that only own the input
// and output buffers (a plugin or FFI boundary with no device allocator of its own),
// and processes whose device memory is fully reserved by another pool, where a fresh
// cudaMalloc would fail and cudaFree would synchronise the device.  For them the
// backward's scratch (fp32 dQ accumulator + Delta) lives in this fixed array, which
// every GPU that loads the library holds until the process exits.
namespace {

constexpr size_t kNoAllocScratchBytes = FA4D_BWD_NOALLOC_MAX_WORKSPACE;  // per device

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device.  In host code the
// symbol is only a stand-in, so the address is looked up once per device (with that
// device current) and cached.
void* noalloc_scratch_ptr(int* err) {
  static std::mutex mu;
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    *err = fail(FA4D_ERR_CUDA, "no current device for the scratch lookup");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      *err = fail(FA4D_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed on device %d: %s", dev,
                  cudaGetErrorString(e));
      return nullptr;
    }
    ptrs[dev] = p;
  }
  return ptrs[dev];
}

}  // namespace

extern "C" {

int fa4d_bwd_noalloc(const fa4d_bwd_args* a, void* stream) {
  if (!a) return fail(FA4D_ERR_INVALID, "args is NULL");
  int rc = check_common(a->B, a->Tq, a->Tk, a->Hq, a->Hk, a->D, a->dtype, a->causal, a->scale);
  if (rc) return rc;
  const size_t need = fa4d_bwd_workspace_size(a->B, a->Tq, a->Hq, a->D);
  if (need > kNoAllocScratchBytes)
    return fail(FA4D_ERR_WORKSPACE,
                "fa4d_bwd_noalloc: this problem needs %zu bytes of scratch but the built-in buffer holds %zu "
                "(B*Tq*Hq*D*4 plus Delta); use fa4d_bwd with a caller-owned workspace",
                need, kNoAllocScratchBytes);
  if (!a->q) return fail(FA4D_ERR_INVALID, "q is NULL");
  if ((rc = bind_device_of(a->q, "q"))) return rc;
  void* scratch = noalloc_scratch_ptr(&rc);
  if (!scratch) return rc;
  fa4d_bwd_args b = *a;
  b.workspace = scratch;
  // Sized like fa4d_bwd's basic workspace, so the call runs the same (unsplit) plan.
  b.workspace_bytes = need;
  // The preprocess stage zeroes the dQ accumulator and writes every Delta entry, so
  // nothing left in the buffer by an earlier call reaches this one's results.
  return bwd_stages(&b, 0, 2, stream);
}

}  // extern "C"
