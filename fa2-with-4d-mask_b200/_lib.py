"""ctypes binding of libfa4d.so (the C ABI in include/fa4d.h) plus the tensor
plumbing the autograd op needs: stride extraction, output/workspace allocation
and stream selection.  PyTorch only supplies device memory and the current
stream; all attention arithmetic runs in the library's sm_100a kernels.

There is no fallback: if the library is missing or cannot be loaded, every entry
point raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libfa4d.so"

FA4D_BF16 = 0
FA4D_F16 = 1
CAUSAL_NONE = 0
CAUSAL_TOP_LEFT = 1
CAUSAL_BOTTOM_RIGHT = 2

FA4D_OK = 0
FA4D_ERR_INVALID = -1
FA4D_ERR_UNSUPPORTED = -2
FA4D_ERR_CUDA = -3
FA4D_ERR_DRIVER = -4
FA4D_ERR_LAYOUT = -5
FA4D_ERR_WORKSPACE = -6

EXPORTED_SYMBOLS = (
    "fa4d_lse_row_stride",
    "fa4d_bwd_workspace_size",
    "fa4d_fwd",
    "fa4d_bwd",
    "fa4d_bwd_preprocess",
    "fa4d_bwd_main",
    "fa4d_bwd_dq_convert",
    "fa4d_bwd_noalloc",
    "fa4d_last_error",
    "fa4d_device_status",
    "fa4d_abi_version",
    "fa4d_check_exp2",
    "fa4d_mask_blocks",
    "fa4d_mask_blocks_size",
    "fa4d_mask_prepare",
    "fa4d_mask_prepare_size",
    "fa4d_check_wait_timeout",
    "fa4d_bwd_workspace_size_ex",
    "fa4d_bwd_group_split",
    "fa4d_mask_prepare_docs",
)
DEV_TIMEOUT_FWD, DEV_TIMEOUT_BWD, DEV_TIMEOUT_CHECK = 1, 2, 4

ABI_VERSION = 2
BLOCK = 128  # rows / keys per block of the mask's block map
BLOCK_EMPTY, BLOCK_PARTIAL, BLOCK_FULL = 0, 1, 2

_i64x3 = ctypes.c_int64 * 3


class FwdArgs(ctypes.Structure):
    """Mirror of ``fa4d_fwd_args``."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("mask", ctypes.c_void_p),
        ("score", ctypes.c_void_p),
        ("q_stride", _i64x3),
        ("k_stride", _i64x3),
        ("v_stride", _i64x3),
        ("o_stride", _i64x3),
        ("mask_stride", _i64x3),
        ("score_stride", _i64x3),
        ("B", ctypes.c_int32),
        ("Tq", ctypes.c_int32),
        ("Tk", ctypes.c_int32),
        ("Hq", ctypes.c_int32),
        ("Hk", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("causal", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("reserved", ctypes.c_int32 * 3),
        ("mask_blocks", ctypes.c_void_p),
        ("mask_blocks_stride", ctypes.c_int64 * 2),
        ("mask_prepared", ctypes.c_void_p),
    ]


class BwdArgs(ctypes.Structure):
    """Mirror of ``fa4d_bwd_args``."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("dout", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("mask", ctypes.c_void_p),
        ("score", ctypes.c_void_p),
        ("dq", ctypes.c_void_p),
        ("dk", ctypes.c_void_p),
        ("dv", ctypes.c_void_p),
        ("q_stride", _i64x3),
        ("k_stride", _i64x3),
        ("v_stride", _i64x3),
        ("o_stride", _i64x3),
        ("do_stride", _i64x3),
        ("dq_stride", _i64x3),
        ("dk_stride", _i64x3),
        ("dv_stride", _i64x3),
        ("mask_stride", _i64x3),
        ("score_stride", _i64x3),
        ("B", ctypes.c_int32),
        ("Tq", ctypes.c_int32),
        ("Tk", ctypes.c_int32),
        ("Hq", ctypes.c_int32),
        ("Hk", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("causal", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("deterministic", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("mask_blocks", ctypes.c_void_p),
        ("mask_blocks_stride", ctypes.c_int64 * 2),
        ("mask_prepared", ctypes.c_void_p),
    ]


_LIB: Optional[ctypes.CDLL] = None


def load_library(path: Optional[os.PathLike] = None) -> ctypes.CDLL:
    """Loads libfa4d.so once and declares the prototypes of include/fa4d.h."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: build it with `python {HERE / 'build.py'}` "
            "(the attention op has no fallback implementation)"
        )
    lib = ctypes.CDLL(str(p))
    lib.fa4d_lse_row_stride.argtypes = [ctypes.c_int32]
    lib.fa4d_lse_row_stride.restype = ctypes.c_int64
    lib.fa4d_bwd_workspace_size.argtypes = [ctypes.c_int32] * 4
    lib.fa4d_bwd_workspace_size.restype = ctypes.c_size_t
    lib.fa4d_bwd_workspace_size_ex.argtypes = [ctypes.c_int32] * 6
    lib.fa4d_bwd_workspace_size_ex.restype = ctypes.c_size_t
    lib.fa4d_bwd_group_split.argtypes = [ctypes.c_int32] * 7
    lib.fa4d_bwd_group_split.restype = ctypes.c_int32
    lib.fa4d_fwd.argtypes = [ctypes.POINTER(FwdArgs), ctypes.c_void_p]
    lib.fa4d_fwd.restype = ctypes.c_int
    for name in ("fa4d_bwd", "fa4d_bwd_preprocess", "fa4d_bwd_main", "fa4d_bwd_dq_convert", "fa4d_bwd_noalloc"):
        fn = getattr(lib, name)
        fn.argtypes = [ctypes.POINTER(BwdArgs), ctypes.c_void_p]
        fn.restype = ctypes.c_int
    lib.fa4d_last_error.argtypes = []
    lib.fa4d_last_error.restype = ctypes.c_char_p
    lib.fa4d_device_status.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
    lib.fa4d_device_status.restype = ctypes.c_int
    lib.fa4d_abi_version.argtypes = []
    lib.fa4d_abi_version.restype = ctypes.c_int
    lib.fa4d_check_exp2.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_float, ctypes.c_float, ctypes.c_void_p]
    lib.fa4d_check_exp2.restype = ctypes.c_int
    lib.fa4d_mask_blocks_size.argtypes = [ctypes.c_int32] * 4
    lib.fa4d_mask_blocks_size.restype = ctypes.c_size_t
    lib.fa4d_mask_blocks.argtypes = [
        ctypes.c_void_p,
        ctypes.POINTER(ctypes.c_int64),
        ctypes.c_int32,
        ctypes.c_int32,
        ctypes.c_int32,
        ctypes.c_int32,
        ctypes.c_void_p,
        ctypes.c_void_p,
    ]
    lib.fa4d_mask_blocks.restype = ctypes.c_int
    lib.fa4d_check_wait_timeout.argtypes = [ctypes.c_int, ctypes.c_int64, ctypes.c_void_p]
    lib.fa4d_check_wait_timeout.restype = ctypes.c_int
    lib.fa4d_mask_prepare_size.argtypes = [ctypes.c_int32] * 4
    lib.fa4d_mask_prepare_size.restype = ctypes.c_size_t
    lib.fa4d_mask_prepare.argtypes = lib.fa4d_mask_blocks.argtypes
    lib.fa4d_mask_prepare.restype = ctypes.c_int
    lib.fa4d_mask_prepare_docs.argtypes = [
        ctypes.c_void_p,
        ctypes.c_void_p,
        ctypes.POINTER(ctypes.c_int64),
        ctypes.c_int32,
        ctypes.c_int32,
        ctypes.c_int32,
        ctypes.c_void_p,
        ctypes.c_void_p,
    ]
    lib.fa4d_mask_prepare_docs.restype = ctypes.c_int
    version = lib.fa4d_abi_version()
    if version != ABI_VERSION:
        raise RuntimeError(f"{p}: ABI version {version}, expected {ABI_VERSION}; rebuild with build.py")
    if path is None:
        _LIB = lib
    return lib


class LayoutError(ValueError):
    """Raised when a tensor's strides cannot be read by TMA (caller may copy and retry)."""


def _raise(lib: ctypes.CDLL, rc: int, what: str) -> None:
    msg = (lib.fa4d_last_error() or b"").decode(errors="replace")
    text = f"{what}: {msg} (code {rc})"
    if rc == FA4D_ERR_LAYOUT:
        raise LayoutError(text)
    if rc in (FA4D_ERR_INVALID, FA4D_ERR_UNSUPPORTED, FA4D_ERR_WORKSPACE):
        raise ValueError(text)
    raise RuntimeError(text)


def _dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return FA4D_BF16
    if dt == torch.float16:
        return FA4D_F16
    raise ValueError(f"unsupported dtype {dt}: expected bf16 or fp16")


def _bth_strides(x: torch.Tensor) -> tuple:
    """(batch, seq, head) element strides of a [B, T, H, D] view."""
    return (x.stride(0), x.stride(1), x.stride(2))


def _bias_strides(x: Optional[torch.Tensor]) -> tuple:
    """(batch, head, row) strides of a [B|1, H|1, Tq, Tk] tensor; broadcast dims get 0."""
    if x is None:
        return (0, 0, 0)
    sb = 0 if x.shape[0] == 1 else x.stride(0)
    sh = 0 if x.shape[1] == 1 else x.stride(1)
    return (sb, sh, x.stride(2))


def tma_friendly(x: torch.Tensor) -> bool:
    """True if a [B, T, H, D] 16-bit view can be described by a TMA tensor map."""
    if x.stride(3) != 1 or x.data_ptr() % 16 != 0:
        return False
    for dim in range(3):
        if x.shape[dim] != 1 and (x.stride(dim) <= 0 or x.stride(dim) % 8 != 0):
            return False
    return True


def as_tma(x: torch.Tensor) -> torch.Tensor:
    return x if tma_friendly(x) else x.contiguous()


def prepare_bias(x: Optional[torch.Tensor], dtype: torch.dtype) -> Optional[torch.Tensor]:
    """Mask/score as the kernel reads them: given dtype, unit key stride (broadcast views kept)."""
    if x is None:
        return None
    if x.dtype != dtype:
        x = x.to(dtype)
    if x.stride(3) != 1:
        x = x.contiguous()
    return x


class BlockMap:
    """Block map of one mask (``fa4d_mask_blocks``): ``blocks`` is a uint8 tensor
    [Bm, Hm, ceil(Tq/128), ceil(Tk/128)] and ``strides`` the (batch, head) byte
    strides the kernels index it with (0 where the mask broadcasts)."""

    __slots__ = ("blocks", "strides")

    def __init__(self, blocks: torch.Tensor, strides: tuple):
        self.blocks = blocks
        self.strides = strides

    def counts(self) -> dict:
        """Number of EMPTY / PARTIAL / FULL blocks (synchronises)."""
        flat = self.blocks.flatten().to(torch.int64)
        c = torch.bincount(flat, minlength=3).tolist()
        return {"empty": c[0], "partial": c[1], "full": c[2]}


def mask_blocks(mask: torch.Tensor) -> BlockMap:
    """Runs the block-occupancy pre-pass over a [B|1, H|1, Tq, Tk] bool/uint8 mask view
    with unit key stride (broadcast dimensions may have stride 0)."""
    lib = load_library()
    if mask.dim() != 4 or mask.element_size() != 1 or mask.stride(3) != 1:
        raise ValueError("mask must be a 4D bool/uint8 tensor with unit key stride")
    Bf, Hf, Tq, Tk = mask.shape
    sb, sh, sr = _bias_strides(mask)
    Bm = Bf if sb != 0 else 1
    Hm = Hf if sh != 0 else 1
    nqb, nkb = -(-Tq // BLOCK), -(-Tk // BLOCK)
    blocks = torch.empty((Bm, Hm, nqb, nkb), dtype=torch.uint8, device=mask.device)
    st = (ctypes.c_int64 * 3)(sb, sh, sr)
    with torch.cuda.device(mask.device):
        rc = lib.fa4d_mask_blocks(mask.data_ptr(), st, Bm, Hm, Tq, Tk, blocks.data_ptr(), _stream_ptr(mask.device))
    if rc != FA4D_OK:
        _raise(lib, rc, "fa4d_mask_blocks")
    strides = (Hm * nqb * nkb if Bm > 1 else 0, nqb * nkb if Hm > 1 else 0)
    return BlockMap(blocks, strides)


class PreparedMask:
    """Output of ``fa4d_mask_prepare`` for one mask: the block map and the mask as
    packed bits (forward row layout, backward column layout) in one device buffer."""

    __slots__ = ("buffer", "Bm", "Hm", "Tq", "Tk")

    def __init__(self, buffer: torch.Tensor, Bm: int, Hm: int, Tq: int, Tk: int):
        self.buffer = buffer
        self.Bm, self.Hm, self.Tq, self.Tk = Bm, Hm, Tq, Tk

    @property
    def nqb(self) -> int:
        return -(-self.Tq // BLOCK)

    @property
    def nkb(self) -> int:
        return -(-self.Tk // BLOCK)

    def _offsets(self) -> tuple:
        a = lambda x: -(-x // 256) * 256
        bh = self.Bm * self.Hm
        nqt = -(-self.Tq // 64)
        row = a(bh * self.nqb * self.nkb)
        col = row + a(bh * self.nkb * self.Tq * 16)
        return row, col, nqt

    def kb_order(self) -> torch.Tensor:
        """Key-tile order view [Bm, Hm, nkb] (int32): key tiles by decreasing number of
        non-EMPTY query blocks, the order the backward launches them in."""
        _, col, nqt = self._offsets()
        off = col + -(-(self.Bm * self.Hm * nqt * self.Tk * 8) // 256) * 256
        n = self.Bm * self.Hm * self.nkb * 4
        return self.buffer[off : off + n].view(torch.int32).view(self.Bm, self.Hm, self.nkb)

    def blocks(self) -> torch.Tensor:
        """Block map view [Bm, Hm, nqb, nkb] (uint8)."""
        n = self.Bm * self.Hm * self.nqb * self.nkb
        return self.buffer[:n].view(self.Bm, self.Hm, self.nqb, self.nkb)

    def row_bits(self) -> torch.Tensor:
        """Row bits view [Bm, Hm, nkb, Tq, 4] (int32 words)."""
        row, _, _ = self._offsets()
        n = self.Bm * self.Hm * self.nkb * self.Tq * 16
        return self.buffer[row : row + n].view(torch.int32).view(self.Bm, self.Hm, self.nkb, self.Tq, 4)

    def col_bits(self) -> torch.Tensor:
        """Column bits view [Bm, Hm, nqt, Tk, 2] (int32 words)."""
        _, col, nqt = self._offsets()
        n = self.Bm * self.Hm * nqt * self.Tk * 8
        return self.buffer[col : col + n].view(torch.int32).view(self.Bm, self.Hm, nqt, self.Tk, 2)


def mask_prepare(mask: torch.Tensor) -> PreparedMask:
    """Runs ``fa4d_mask_prepare`` over a [B|1, H|1, Tq, Tk] bool/uint8 mask view with
    unit key stride (broadcast dimensions may have stride 0)."""
    lib = load_library()
    if mask.dim() != 4 or mask.element_size() != 1 or mask.stride(3) != 1:
        raise ValueError("mask must be a 4D bool/uint8 tensor with unit key stride")
    Bf, Hf, Tq, Tk = mask.shape
    sb, sh, sr = _bias_strides(mask)
    Bm = Bf if sb != 0 else 1
    Hm = Hf if sh != 0 else 1
    nbytes = int(lib.fa4d_mask_prepare_size(Bm, Hm, Tq, Tk))
    buf = torch.empty((nbytes,), dtype=torch.uint8, device=mask.device)
    st = (ctypes.c_int64 * 3)(sb, sh, sr)
    with torch.cuda.device(mask.device):
        rc = lib.fa4d_mask_prepare(mask.data_ptr(), st, Bm, Hm, Tq, Tk, buf.data_ptr(), _stream_ptr(mask.device))
    if rc != FA4D_OK:
        _raise(lib, rc, "fa4d_mask_prepare")
    return PreparedMask(buf, Bm, Hm, Tq, Tk)


def mask_prepare_docs(doc_q: torch.Tensor, doc_k: torch.Tensor, batch: int) -> PreparedMask:
    """Runs ``fa4d_mask_prepare_docs``: the prepared mask of per-token document ids
    doc_q [B|1, Tq] and doc_k [B|1, Tk] (keep iff equal and >= 0), for batch ``batch``."""
    lib = load_library()
    if doc_q.dim() != 2 or doc_k.dim() != 2:
        raise ValueError("document ids must be [B or 1, T] tensors")
    doc_q = doc_q.to(torch.int32)
    doc_k = doc_k.to(torch.int32)
    if doc_q.stride(1) != 1:
        doc_q = doc_q.contiguous()
    if doc_k.stride(1) != 1:
        doc_k = doc_k.contiguous()
    Tq, Tk = doc_q.shape[1], doc_k.shape[1]
    st = (ctypes.c_int64 * 2)(0 if doc_q.shape[0] == 1 else doc_q.stride(0), 0 if doc_k.shape[0] == 1 else doc_k.stride(0))
    nbytes = int(lib.fa4d_mask_prepare_size(batch, 1, Tq, Tk))
    buf = torch.empty((nbytes,), dtype=torch.uint8, device=doc_q.device)
    with torch.cuda.device(doc_q.device):
        rc = lib.fa4d_mask_prepare_docs(doc_q.data_ptr(), doc_k.data_ptr(), st, batch, Tq, Tk, buf.data_ptr(),
                                        _stream_ptr(doc_q.device))
    if rc != FA4D_OK:
        _raise(lib, rc, "fa4d_mask_prepare_docs")
    return PreparedMask(buf, batch, 1, Tq, Tk)


def _set_blocks(a, mask: Optional[torch.Tensor], blocks) -> None:
    """Attaches a BlockMap (map only) or a PreparedMask (map + bits) to the args; a
    PreparedMask without a mask tensor is a document-id preparation."""
    a.mask_blocks = None
    a.mask_prepared = None
    if blocks is None:
        return
    if isinstance(blocks, PreparedMask):
        a.mask_prepared = blocks.buffer.data_ptr()
    elif mask is None:
        return
    else:
        a.mask_blocks = blocks.blocks.data_ptr()
        a.mask_blocks_stride = (ctypes.c_int64 * 2)(*blocks.strides)


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def lse_row_stride(Tq: int) -> int:
    return int(load_library().fa4d_lse_row_stride(int(Tq)))


def forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    mask: Optional[torch.Tensor],
    score: Optional[torch.Tensor],
    scale: float,
    causal: int,
    blocks=None,
    out: Optional[torch.Tensor] = None,
) -> tuple:
    """Runs fa4d_fwd (with the mask's BlockMap or PreparedMask when given).  q: [B, Tq, Hq, D] view, k/v: [B, Tk, Hk, D] views (TMA-friendly).
    Returns (O [B, Tq, Hq, D], LSE [B, Hq, lse_row_stride(Tq)] fp32); O is ``out`` when
    given (any [B, Tq, Hq, D] view with 16-byte aligned rows), else a new tensor."""
    lib = load_library()
    B, Tq, Hq, D = q.shape
    Tk, Hk = k.shape[1], k.shape[2]
    if out is not None:
        if tuple(out.shape) != (B, Tq, Hq, D) or out.dtype != q.dtype or out.device != q.device:
            raise ValueError(f"out must be a {q.dtype} tensor of shape {(B, Tq, Hq, D)} on {q.device}")
        o = out
    else:
        o = torch.empty((B, Tq, Hq, D), dtype=q.dtype, device=q.device)
    lse = torch.empty((B, Hq, lse_row_stride(Tq)), dtype=torch.float32, device=q.device)
    a = FwdArgs()
    a.q, a.k, a.v, a.o, a.lse = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr()
    a.mask = mask.data_ptr() if mask is not None else None
    a.score = score.data_ptr() if score is not None else None
    a.q_stride = _i64x3(*_bth_strides(q))
    a.k_stride = _i64x3(*_bth_strides(k))
    a.v_stride = _i64x3(*_bth_strides(v))
    a.o_stride = _i64x3(*_bth_strides(o))
    a.mask_stride = _i64x3(*_bias_strides(mask))
    a.score_stride = _i64x3(*_bias_strides(score))
    a.B, a.Tq, a.Tk, a.Hq, a.Hk, a.D = B, Tq, Tk, Hq, Hk, D
    a.dtype = _dtype_code(q.dtype)
    a.causal = int(causal)
    a.scale = float(scale)
    _set_blocks(a, mask, blocks)
    with torch.cuda.device(q.device):
        rc = lib.fa4d_fwd(ctypes.byref(a), _stream_ptr(q.device))
    if rc != FA4D_OK:
        _raise(lib, rc, "fa4d_fwd")
    return o, lse


def backward(
    dout: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    o: torch.Tensor,
    lse: torch.Tensor,
    mask: Optional[torch.Tensor],
    score: Optional[torch.Tensor],
    scale: float,
    causal: int,
    stages=None,
    blocks=None,
    deterministic: bool = False,
    grads: Optional[tuple] = None,
) -> tuple:
    """Runs fa4d_bwd on [B, T, H, D] views.  Returns (dQ, dK, dV) in the input
    dtype, dK/dV summed over the GQA group.

    ``stages`` optionally replaces the single fa4d_bwd call by a list of callables
    ``f(name, launch)``; each receives the stage name ("preprocess", "main",
    "dq_convert") and a zero-argument function that enqueues that stage, so a caller
    can bracket each stage (e.g. with CUDA events).  ``deterministic`` selects the
    bit-reproducible backward (dQ from a separate in-order pass; the third stage
    is then that pass).  ``grads`` optionally gives the (dQ, dK, dV) output views
    to write into (16-byte aligned rows), as ``out`` does for the forward."""
    lib = load_library()
    B, Tq, Hq, D = q.shape
    Tk, Hk = k.shape[1], k.shape[2]
    shapes = ((B, Tq, Hq, D), (B, Tk, Hk, D), (B, Tk, Hk, D))
    if grads is not None:
        for g, shp, name in zip(grads, shapes, ("dq", "dk", "dv")):
            if tuple(g.shape) != shp or g.dtype != q.dtype or g.device != q.device:
                raise ValueError(f"{name} must be a {q.dtype} tensor of shape {shp} on {q.device}")
        dq, dk, dv = grads
    else:
        dq, dk, dv = (torch.empty(shp, dtype=q.dtype, device=q.device) for shp in shapes)
    ws_bytes = int(lib.fa4d_bwd_workspace_size_ex(B, Tq, Tk, Hq, Hk, D))
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=q.device)
    a = BwdArgs()
    a.q, a.k, a.v, a.o, a.dout = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr()
    a.lse = lse.data_ptr()
    a.mask = mask.data_ptr() if mask is not None else None
    a.score = score.data_ptr() if score is not None else None
    a.dq, a.dk, a.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    a.q_stride = _i64x3(*_bth_strides(q))
    a.k_stride = _i64x3(*_bth_strides(k))
    a.v_stride = _i64x3(*_bth_strides(v))
    a.o_stride = _i64x3(*_bth_strides(o))
    a.do_stride = _i64x3(*_bth_strides(dout))
    a.dq_stride = _i64x3(*_bth_strides(dq))
    a.dk_stride = _i64x3(*_bth_strides(dk))
    a.dv_stride = _i64x3(*_bth_strides(dv))
    a.mask_stride = _i64x3(*_bias_strides(mask))
    a.score_stride = _i64x3(*_bias_strides(score))
    a.B, a.Tq, a.Tk, a.Hq, a.Hk, a.D = B, Tq, Tk, Hq, Hk, D
    a.dtype = _dtype_code(q.dtype)
    a.causal = int(causal)
    a.scale = float(scale)
    a.deterministic = 1 if deterministic else 0
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws_bytes
    _set_blocks(a, mask, blocks)
    with torch.cuda.device(q.device):
        stream = _stream_ptr(q.device)
        if stages is None:
            rc = lib.fa4d_bwd(ctypes.byref(a), stream)
            if rc != FA4D_OK:
                _raise(lib, rc, "fa4d_bwd")
        else:
            for name in ("preprocess", "main", "dq_convert"):
                fn = getattr(lib, "fa4d_bwd_" + name)

                def launch(fn=fn, name=name):
                    rc = fn(ctypes.byref(a), stream)
                    if rc != FA4D_OK:
                        _raise(lib, rc, "fa4d_bwd_" + name)

                stages(name, launch)
    return dq, dk, dv


def device_status(device: Optional[torch.device] = None, clear: bool = True) -> int:
    """Synchronises the current stream and returns the kernels' timeout bits (0 = none)."""
    lib = load_library()
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(device):
        rc = lib.fa4d_device_status(device.index, _stream_ptr(device), 1 if clear else 0)
    if rc < 0:
        _raise(lib, rc, "fa4d_device_status")
    return rc
