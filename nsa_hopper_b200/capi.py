"""ctypes binding of the C ABI in include/nsa_sel.h (libnsa_sel.so, built in-tree).

This is the reference-facing boundary: the same entry points a cgo/JNI/ctypes host of the
reference's ``forward(Q,K,V,sel,l_prime,BQ,cyc)`` op (nsa_v2.cu:147-170) would bind.  Device
buffers are passed as raw pointers (e.g. ``tensor.data_ptr()``), streams as raw handles
(``torch.cuda.current_stream().cuda_stream``).  Loading fails loudly when the library is
missing: there is no fallback path.
"""
from __future__ import annotations

import ctypes
import os
import re
from typing import Dict, List, Optional

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
LIB_PATH = os.path.join(PKG_DIR, "libnsa_sel.so")
HEADER_PATH = os.path.join(REPO_DIR, "include", "nsa_sel.h")

NSA_OK = 0
NSA_ERR_INVALID_ARG = -1
NSA_ERR_UNSUPPORTED = -2
NSA_ERR_CUDA = -3
NSA_ERR_DRIVER = -4
NSA_DEVERR_TIMEOUT = 1
NSA_DEBUG_STALL = 1
NSA_DEBUG_STATIC_UNITS = 2
NSA_DEBUG_NO_ROW_OWNER = 4
NSA_DEBUG_RO_PAD128 = 8
DTYPE_BF16 = 0
DTYPE_F32 = 1
KEYMAP_CAUSAL = 0
KEYMAP_COMPRESSED = 1


class NsaSelDesc(ctypes.Structure):
    """Mirror of ``nsa_sel_desc``."""

    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("sel", ctypes.c_void_p), ("cu_seqlens", ctypes.c_void_p),
        ("o", ctypes.c_void_p), ("lse", ctypes.c_void_p), ("cyc", ctypes.c_void_p), ("err", ctypes.c_void_p),
        ("batch", ctypes.c_int32), ("heads_q", ctypes.c_int32), ("heads_kv", ctypes.c_int32),
        ("seq_len", ctypes.c_int32), ("d_qk", ctypes.c_int32), ("d_v", ctypes.c_int32),
        ("n_qblocks", ctypes.c_int32), ("n_sel", ctypes.c_int32), ("block_size", ctypes.c_int32),
        ("q_block", ctypes.c_int32), ("n_seqs", ctypes.c_int32), ("o_dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("bkv_begin", ctypes.c_int32), ("bkv_end", ctypes.c_int32),
        ("qb_begin", ctypes.c_int32), ("qb_end", ctypes.c_int32),
        ("timeout_ms", ctypes.c_int32), ("max_ctas", ctypes.c_int32), ("debug_flags", ctypes.c_int32),
        ("kv_len", ctypes.c_int32),
        ("window", ctypes.c_int32),
        ("key_map", ctypes.c_int32),
        ("o_accumulate", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("o_weight", ctypes.c_void_p),
    ]


class NsaSelPlanInfo(ctypes.Structure):
    """Mirror of ``nsa_sel_plan_info``."""

    _fields_ = [
        ("n_cols", ctypes.c_int32), ("q_per_unit", ctypes.c_int32), ("parts", ctypes.c_int32),
        ("n_units", ctypes.c_int32), ("k_stages", ctypes.c_int32), ("v_stages", ctypes.c_int32),
        ("smem_bytes", ctypes.c_int32), ("grid", ctypes.c_int32), ("tmem_cols", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 7),
    ]


class NsaSelHostIO(ctypes.Structure):
    """Mirror of ``nsa_sel_host_io``."""

    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("sel", ctypes.c_void_p),
        ("o", ctypes.c_void_p), ("lse", ctypes.c_void_p), ("token_slices", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 7),
    ]


class NsaSelBwdDesc(ctypes.Structure):
    """Mirror of ``nsa_sel_bwd_desc``."""

    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("sel", ctypes.c_void_p),
        ("o", ctypes.c_void_p), ("lse", ctypes.c_void_p), ("d_o", ctypes.c_void_p),
        ("dq", ctypes.c_void_p), ("dk", ctypes.c_void_p), ("dv", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("err", ctypes.c_void_p),
        ("batch", ctypes.c_int32), ("heads_q", ctypes.c_int32), ("heads_kv", ctypes.c_int32),
        ("seq_len", ctypes.c_int32), ("d", ctypes.c_int32), ("n_sel", ctypes.c_int32),
        ("block_size", ctypes.c_int32), ("o_dtype", ctypes.c_int32), ("scale", ctypes.c_float),
        ("timeout_ms", ctypes.c_int32), ("max_ctas", ctypes.c_int32), ("reserved", ctypes.c_int32 * 5),
    ]


class NsaSelError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"nsa_sel error {code}: {message}")
        self.code = code


_lib = None


def load(path: Optional[str] = None) -> ctypes.CDLL:
    """Load libnsa_sel.so (raises if it has not been built)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise ImportError(f"{p} is missing: run `python -c 'import __graft_entry__ as g; g.build()'` first")
    lib = ctypes.CDLL(p)
    vp, i32 = ctypes.c_void_p, ctypes.c_int32
    lib.nsa_sel_forward.argtypes = [vp, vp, vp, vp, vp, vp] + [i32] * 9 + [vp]
    lib.nsa_sel_forward.restype = ctypes.c_int
    lib.nsa_sel_forward_lse.argtypes = [vp, vp, vp, vp, vp, i32, vp, vp, i32] + [i32] * 10 + [ctypes.c_float, vp]
    lib.nsa_sel_forward_lse.restype = ctypes.c_int
    lib.nsa_sel_run.argtypes = [ctypes.POINTER(NsaSelDesc), vp]
    lib.nsa_sel_run.restype = ctypes.c_int
    if hasattr(lib, "nsa_sel_run_host"):  # absent from builds that predate it
        lib.nsa_sel_run_host.argtypes = [ctypes.POINTER(NsaSelDesc), ctypes.POINTER(NsaSelHostIO), vp]
        lib.nsa_sel_run_host.restype = ctypes.c_int
    lib.nsa_sel_plan.argtypes = [ctypes.POINTER(NsaSelDesc), i32, ctypes.POINTER(NsaSelPlanInfo)]
    lib.nsa_sel_plan.restype = ctypes.c_int
    lib.nsa_sel_last_error.argtypes = []
    lib.nsa_sel_last_error.restype = ctypes.c_char_p
    lib.nsa_sel_version.argtypes = []
    lib.nsa_sel_version.restype = i32
    lib.nsa_sel_select.argtypes = [vp, vp, vp, vp] + [i32] * 9 + [vp]
    lib.nsa_sel_select.restype = ctypes.c_int
    lib.nsa_sel_select_workspace_bytes.argtypes = [i32] * 5
    lib.nsa_sel_select_workspace_bytes.restype = ctypes.c_int64
    lib.nsa_sel_select_noalloc.argtypes = [vp, vp, vp] + [i32] * 9 + [vp]
    lib.nsa_sel_select_noalloc.restype = ctypes.c_int
    lib.nsa_sel_select_static_scratch_bytes.argtypes = []
    lib.nsa_sel_select_static_scratch_bytes.restype = ctypes.c_int64
    lib.nsa_sel_backward_workspace_bytes.argtypes = [ctypes.POINTER(NsaSelBwdDesc)]
    lib.nsa_sel_backward_workspace_bytes.restype = ctypes.c_int64
    lib.nsa_sel_backward.argtypes = [ctypes.POINTER(NsaSelBwdDesc), vp]
    lib.nsa_sel_backward.restype = ctypes.c_int
    lib.nsa_sel_select_status.argtypes = []
    lib.nsa_sel_select_status.restype = ctypes.c_int32
    if path is None:
        _lib = lib
    return lib


def last_error() -> str:
    return load().nsa_sel_last_error().decode()


def check(rc: int) -> None:
    if rc != NSA_OK:
        raise NsaSelError(rc, last_error())


def header_functions(header: str = HEADER_PATH) -> List[str]:
    """Names of the functions declared in include/nsa_sel.h."""
    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(nsa_[a-z_0-9]+)\s*\(", text, flags=re.M)


def make_desc(**kw) -> NsaSelDesc:
    d = NsaSelDesc()
    ctypes.memset(ctypes.addressof(d), 0, ctypes.sizeof(d))
    for key, val in kw.items():
        if not hasattr(d, key):
            raise KeyError(key)
        setattr(d, key, val)
    return d


def run(desc: NsaSelDesc, stream: int = 0) -> None:
    check(load().nsa_sel_run(ctypes.byref(desc), ctypes.c_void_p(stream)))


def plan(desc: NsaSelDesc, sm_count: int = 148) -> Dict[str, int]:
    info = NsaSelPlanInfo()
    check(load().nsa_sel_plan(ctypes.byref(desc), sm_count, ctypes.byref(info)))
    return {name: getattr(info, name) for name, _ in NsaSelPlanInfo._fields_ if name != "reserved"}


def select_workspace_bytes(B: int, Hkv: int, T: int, d: int, l_prime: int) -> int:
    return int(load().nsa_sel_select_workspace_bytes(B, Hkv, T, d, l_prime))


def select(q: int, k: int, workspace: int, sel_out: int, B: int, Hq: int, Hkv: int, T: int, d: int, l_prime: int,
           n_sel: int, cmp_block: int = 32, cmp_stride: int = 16, stream: int = 0) -> None:
    """nsa_sel_select on device pointers (see include/nsa_sel.h)."""
    check(load().nsa_sel_select(ctypes.c_void_p(q), ctypes.c_void_p(k), ctypes.c_void_p(workspace),
                                ctypes.c_void_p(sel_out), B, Hq, Hkv, T, d, l_prime, n_sel, cmp_block, cmp_stride,
                                ctypes.c_void_p(stream)))


def select_noalloc(q: int, k: int, sel_out: int, B: int, Hq: int, Hkv: int, T: int, d: int, l_prime: int,
                   n_sel: int, cmp_block: int = 32, cmp_stride: int = 16, stream: int = 0) -> None:
    """nsa_sel_select_noalloc: block selection with the library's static scratch (no allocation)."""
    check(load().nsa_sel_select_noalloc(ctypes.c_void_p(q), ctypes.c_void_p(k), ctypes.c_void_p(sel_out), B, Hq,
                                        Hkv, T, d, l_prime, n_sel, cmp_block, cmp_stride, ctypes.c_void_p(stream)))


def select_status() -> int:
    """nsa_sel_select_status: device error bits of the selection launches so far (then cleared)."""
    return int(load().nsa_sel_select_status())


def make_host_io(**kw) -> NsaSelHostIO:
    io = NsaSelHostIO()
    ctypes.memset(ctypes.addressof(io), 0, ctypes.sizeof(io))
    for key, val in kw.items():
        if not hasattr(io, key):
            raise KeyError(key)
        setattr(io, key, val)
    return io


def run_host(desc: NsaSelDesc, io: NsaSelHostIO, stream: int = 0) -> None:
    """nsa_sel_run_host: host inputs in, host outputs back, copies pipelined with the kernel."""
    check(load().nsa_sel_run_host(ctypes.byref(desc), ctypes.byref(io), ctypes.c_void_p(stream)))


def make_bwd_desc(**kw) -> NsaSelBwdDesc:
    d = NsaSelBwdDesc()
    ctypes.memset(ctypes.addressof(d), 0, ctypes.sizeof(d))
    for key, val in kw.items():
        if not hasattr(d, key):
            raise KeyError(key)
        setattr(d, key, val)
    return d


def backward_workspace_bytes(desc: NsaSelBwdDesc) -> int:
    """nsa_sel_backward_workspace_bytes (raises on an invalid description)."""
    n = int(load().nsa_sel_backward_workspace_bytes(ctypes.byref(desc)))
    if n < 0:
        raise NsaSelError(NSA_ERR_INVALID_ARG, last_error())
    return n


def backward(desc: NsaSelBwdDesc, stream: int = 0) -> None:
    """nsa_sel_backward: adds dQ, dK, dV of the selected branch (see include/nsa_sel.h)."""
    check(load().nsa_sel_backward(ctypes.byref(desc), ctypes.c_void_p(stream)))
