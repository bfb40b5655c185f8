"""ctypes binding of libpalu_b200.so (the C ABI in include/palu_b200.h).

The shared library is built in-tree (``palu_b200.build.build()``) and loaded from this package's
directory. There is no fallback: if the library or a CUDA device is missing, every call raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_NAME = "libpalu_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

PALU_OK, PALU_ERR_INVALID, PALU_ERR_WORKSPACE, PALU_ERR_CUDA = 0, 1, 2, 3
PALU_BF16, PALU_F32 = 0, 1

# Every symbol include/palu_b200.h declares (checked by the CPU test suite).
EXPORTED = ("palu_decode_attn", "palu_decode_attn_static", "palu_decode_attn_paged", "palu_append_latents_paged",
            "palu_rope_q_append", "palu_add_rms_norm", "palu_swiglu",
            "palu_workspace_bytes", "palu_choose_splits", "palu_append_latents",
            "palu_plain_gqa_decode", "palu_pack_cs_table", "palu_set_kernel", "palu_set_rope_mode", "palu_kernel_for",
            "palu_read_status",
            "palu_set_wait_limit", "palu_decode_attn_f8", "palu_quantize_latents_f8", "palu_append_latents_f8",
            "palu_decode_attn_f4", "palu_quantize_latents_f4", "palu_append_latents_f4",
            "palu_last_error", "palu_version")
PALU_KERNEL_AUTO, PALU_KERNEL_MMA, PALU_KERNEL_TC = 0, 1, 2
PALU_ROPE_ABSOLUTE, PALU_ROPE_CHUNK_RELATIVE = 0, 1


class DecodeDims(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("n_q_heads", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32),
                ("n_groups", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("r_k", ctypes.c_int32),
                ("r_v", ctypes.c_int32), ("max_seq", ctypes.c_int32), ("splits", ctypes.c_int32)]


class PageTable(ctypes.Structure):
    _fields_ = [("table", ctypes.c_void_p), ("table_ld", ctypes.c_int32), ("block_size", ctypes.c_int32),
                ("n_blocks", ctypes.c_int32)]


_lib = None


def load() -> ctypes.CDLL:
    """Load the library (once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_NAME} is not built: run palu_b200.build.build() (looked in {LIB_PATH.parent})")
    lib = ctypes.CDLL(str(LIB_PATH))
    vp, i32, i64, sz, f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float
    dims_p = ctypes.POINTER(DecodeDims)
    lib.palu_decode_attn.argtypes = [vp, vp, vp, vp, i64, vp, vp, vp, vp, i32, vp, sz, dims_p, f32, vp]
    lib.palu_decode_attn.restype = ctypes.c_int
    lib.palu_decode_attn_static.argtypes = [vp, vp, vp, vp, i64, vp, vp, vp, vp, i32, dims_p, f32, vp]
    lib.palu_decode_attn_static.restype = ctypes.c_int
    lib.palu_decode_attn_f8.argtypes = [vp, vp, vp, vp, vp, vp, i64, vp, vp, vp, vp, i32, vp, sz, dims_p, f32, vp]
    lib.palu_decode_attn_f8.restype = ctypes.c_int
    lib.palu_quantize_latents_f8.argtypes = [vp, i64, i32, vp, vp, vp]
    lib.palu_quantize_latents_f8.restype = ctypes.c_int
    lib.palu_append_latents_f8.argtypes = [vp, vp, vp, vp, vp, vp, vp, dims_p, vp]
    lib.palu_append_latents_f8.restype = ctypes.c_int
    for f in ("f4",):
        getattr(lib, f"palu_decode_attn_{f}").argtypes = lib.palu_decode_attn_f8.argtypes
        getattr(lib, f"palu_decode_attn_{f}").restype = ctypes.c_int
        getattr(lib, f"palu_quantize_latents_{f}").argtypes = lib.palu_quantize_latents_f8.argtypes
        getattr(lib, f"palu_quantize_latents_{f}").restype = ctypes.c_int
        getattr(lib, f"palu_append_latents_{f}").argtypes = lib.palu_append_latents_f8.argtypes
        getattr(lib, f"palu_append_latents_{f}").restype = ctypes.c_int
    pages_p = ctypes.POINTER(PageTable)
    lib.palu_decode_attn_paged.argtypes = [vp, vp, vp, vp, i64, vp, vp, vp, pages_p, vp, i32, vp, sz, dims_p, f32, vp]
    lib.palu_decode_attn_paged.restype = ctypes.c_int
    lib.palu_append_latents_paged.argtypes = [vp, vp, vp, pages_p, vp, vp, dims_p, vp]
    lib.palu_append_latents_paged.restype = ctypes.c_int
    lib.palu_rope_q_append.argtypes = [vp, i64, i32, vp, vp, vp, vp, vp, vp, pages_p, dims_p, vp]
    lib.palu_rope_q_append.restype = ctypes.c_int
    lib.palu_add_rms_norm.argtypes = [vp, vp, i32, vp, vp, i32, i32, f32, vp]
    lib.palu_add_rms_norm.restype = ctypes.c_int
    lib.palu_swiglu.argtypes = [vp, i64, i32, vp, i32, vp]
    lib.palu_swiglu.restype = ctypes.c_int
    lib.palu_plain_gqa_decode.argtypes = [vp, vp, vp, vp, vp, i32, vp, sz, dims_p, f32, vp]
    lib.palu_plain_gqa_decode.restype = ctypes.c_int
    lib.palu_workspace_bytes.argtypes = [dims_p]
    lib.palu_workspace_bytes.restype = sz
    lib.palu_choose_splits.argtypes = [dims_p]
    lib.palu_choose_splits.restype = i32
    lib.palu_append_latents.argtypes = [vp, vp, vp, vp, vp, dims_p, vp]
    lib.palu_append_latents.restype = ctypes.c_int
    lib.palu_pack_cs_table.argtypes = [vp, i64, i32, vp, i32, vp]
    lib.palu_pack_cs_table.restype = ctypes.c_int
    lib.palu_set_kernel.argtypes = [i32]
    lib.palu_set_kernel.restype = ctypes.c_int
    lib.palu_set_rope_mode.argtypes = [i32]
    lib.palu_set_rope_mode.restype = ctypes.c_int
    lib.palu_set_wait_limit.argtypes = [i64, i32]
    lib.palu_set_wait_limit.restype = ctypes.c_int
    lib.palu_kernel_for.argtypes = [dims_p]
    lib.palu_kernel_for.restype = i32
    lib.palu_read_status.argtypes = [vp, ctypes.POINTER(i32), vp]
    lib.palu_read_status.restype = ctypes.c_int
    lib.palu_last_error.argtypes = []
    lib.palu_last_error.restype = ctypes.c_char_p
    lib.palu_version.argtypes = []
    lib.palu_version.restype = ctypes.c_char_p
    _lib = lib
    return lib


def check(status: int) -> None:
    """Map a nonzero status to RuntimeError carrying palu_last_error()."""
    if status != PALU_OK:
        msg = load().palu_last_error().decode(errors="replace")
        raise RuntimeError(f"palu_b200 error {status}: {msg}")


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("palu_b200 runs on CUDA tensors only (no CPU path); got a tensor on "
                               f"{t.device}")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device) -> int:
    """The raw handle of the current stream on ``device`` (the decode step's host path calls this every
    step: the direct lookup costs well under a microsecond, torch.cuda.current_stream several)."""
    if _RAW_STREAM is not None:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return _RAW_STREAM(idx)
    return torch.cuda.current_stream(device).cuda_stream


_DIMS_CACHE: dict = {}


def dims(batch, n_q, n_kv, n_groups, r_k, r_v, max_seq, splits=0) -> DecodeDims:
    """The DecodeDims of a shape, built once per shape (the library only reads it)."""
    key = (batch, n_q, n_kv, n_groups, r_k, r_v, max_seq, splits)
    d = _DIMS_CACHE.get(key)
    if d is None:
        if len(_DIMS_CACHE) > 256:
            _DIMS_CACHE.clear()
        d = _DIMS_CACHE[key] = DecodeDims(int(batch), int(n_q), int(n_kv), int(n_groups), 128, int(r_k), int(r_v),
                                          int(max_seq), int(splits))
    return d


def pages(table: torch.Tensor, block_size: int, n_blocks: int) -> PageTable:
    """palu_page_table for an int32 [B, table_ld] page table (contiguous rows)."""
    if table.dtype != torch.int32 or table.dim() != 2 or table.stride(1) != 1:
        raise RuntimeError(f"page table must be a row-major int32 [B, blocks per row] tensor, got "
                           f"{table.dtype} {tuple(table.shape)}")
    return PageTable(table.data_ptr(), int(table.stride(0)), int(block_size), int(n_blocks))


_WSB_CACHE: dict = {}


def workspace_bytes(d: DecodeDims) -> int:
    """palu_workspace_bytes(d), cached per shape and kernel choice (set_kernel can change it)."""
    key = (d.batch, d.n_q_heads, d.n_kv_heads, d.n_groups, d.r_k, d.r_v, d.max_seq, d.splits, _KERNEL[0])
    n = _WSB_CACHE.get(key)
    if n is None:
        if len(_WSB_CACHE) > 256:
            _WSB_CACHE.clear()
        n = _WSB_CACHE[key] = int(load().palu_workspace_bytes(ctypes.byref(d)))
    return n


def new_workspace(d: DecodeDims, device) -> torch.Tensor:
    """A zeroed workspace for calls with these dims (the status word at its start must start at 0)."""
    return torch.zeros(workspace_bytes(d), dtype=torch.uint8, device=device)


def choose_splits(d: DecodeDims) -> int:
    return int(load().palu_choose_splits(ctypes.byref(d)))


_KERNEL = [PALU_KERNEL_AUTO]


def set_kernel(which: int) -> None:
    """Choose the decode kernel family (PALU_KERNEL_AUTO / _MMA / _TC) for this process."""
    check(load().palu_set_kernel(int(which)))
    _KERNEL[0] = int(which)


def set_rope_mode(mode: int) -> None:
    """RoPE form of this thread's following decode calls (palu_set_rope_mode, thread-local in the library):
    PALU_ROPE_ABSOLUTE (the reference op's Phase 1) or PALU_ROPE_CHUNK_RELATIVE (its Phase 2). Set on every
    call rather than cached here, so a caller that also uses the C setter directly cannot leave the two out
    of step (about 1 us of host time per decode call)."""
    check(load().palu_set_rope_mode(int(mode)))


def set_wait_limit(wait_ns: int = 0, starve_v: bool = False) -> None:
    """Test hook of the timeout path (palu_set_wait_limit): bound device waits at ``wait_ns`` (0 = the
    default 1 s) and, with ``starve_v``, make a V producer skip its loads so that a wait runs out."""
    check(load().palu_set_wait_limit(int(wait_ns), int(bool(starve_v))))


def kernel_for(d: DecodeDims) -> int:
    return int(load().palu_kernel_for(ctypes.byref(d)))


def read_status(workspace) -> int:
    """The status word a decode call left in ``workspace`` (0 = ok); reading clears it. ``None`` reads the
    static scratch of palu_decode_attn_static on the current device."""
    st = ctypes.c_int32(0)
    if workspace is None:
        check(load().palu_read_status(None, ctypes.byref(st), stream_handle(torch.device("cuda"))))
    else:
        check(load().palu_read_status(workspace.data_ptr(), ctypes.byref(st), stream_handle(workspace.device)))
    return int(st.value)


def env_splits() -> int:
    """Split override for experiments (PALU_SPLITS); 0 = the library's choice."""
    v = os.environ.get("PALU_SPLITS", "").strip()
    return int(v) if v.isdigit() else 0
