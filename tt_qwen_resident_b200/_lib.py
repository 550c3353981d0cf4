"""ctypes binding of libqres.so (include/qres.h); the torch custom ops over it are in ops.py.

The library is built in-tree (``tt_qwen_resident_b200/libqres.so``, see ``build.py``). Nothing here falls back
to another implementation: without the library (or a CUDA device) every entry point raises.
"""
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("QRES_LIB", os.path.join(HERE, "libqres.so"))

QRES_MAX_ROWS = 8
QRES_HIST_SLOTS = 8
QRES_KV_BLOCK = 64
QRES_FLAG_VERIFY = 1
QRES_FLAG_TILE_FINISH = 4
QRES_TOPK = 32
W_GDN_IN, W_ATTN_IN, W_OUT, W_GATEUP, W_DOWN, W_HEAD = range(6)
W_FC = 6  # the MTP draft layer fc
XCHG_NAMES = {0: "none", 1: "nccl", 2: "tagged", 3: "counted"}  # qres_exchange_mode
STATUS = {0: "ok", 1: "bad argument", 2: "CUDA error", 3: "device error", 4: "out of order", 5: "communication"}

# the C-ABI entry points of include/qres.h (checked by tests/test_abi.py)
EXPORTS = [
    "qres_create",
    "qres_destroy",
    "qres_last_error",
    "qres_load_weights",
    "qres_load_gdn_params",
    "qres_load_attn_params",
    "qres_bind_state",
    "qres_load_gdn_state",
    "qres_dump_gdn_state",
    "qres_load_kv",
    "qres_dump_kv",
    "qres_bind_rope",
    "qres_bind_io",
    "qres_bind_sampling",
    "qres_workspace_size",
    "qres_bind_workspace",
    "qres_nccl_unique_id",
    "qres_nccl_init",
    "qres_p2p_window_size",
    "qres_p2p_alloc",
    "qres_p2p_open",
    "qres_exchange_mode",
    "qres_decode_step",
    "qres_capture",
    "qres_replay",
    "qres_release_graph",
    "qres_check",
    "qres_wait_probe",
    "qres_step_launches",
    "qres_gemv_workspace_size",
    "qres_gemv",
    "qres_gdn_mixer",
    "qres_attn_workspace_size",
    "qres_attn_mixer",
    "qres_topk_workspace_size",
    "qres_topk",
    "qres_topk_noalloc",
    "qres_sample",
    "qres_quantize_fp8",
    "qres_tile_weight",
]


class QresError(RuntimeError):
    pass


class Config(ctypes.Structure):
    _fields_ = [
        ("layers", ctypes.c_int32),
        ("attn_interval", ctypes.c_int32),
        ("vocab", ctypes.c_int32),
        ("rows", ctypes.c_int32),
        ("max_pages", ctypes.c_int32),
        ("num_pages", ctypes.c_int32),
        ("sm_count", ctypes.c_int32),
        ("flags", ctypes.c_int32),
    ]


class Weight(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("uscale", ctypes.c_void_p),
        ("rows", ctypes.c_int32),
        ("rows_pad", ctypes.c_int32),
        ("K", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class LayerState(ctypes.Structure):
    _fields_ = [
        ("gdn_state", ctypes.c_void_p),
        ("conv_hist", ctypes.c_void_p),
        ("k_pool", ctypes.c_void_p),
        ("v_pool", ctypes.c_void_p),
    ]


class Io(ctypes.Structure):
    _fields_ = [
        ("tok", ctypes.c_void_p),
        ("x0", ctypes.c_void_p),
        ("embed", ctypes.c_void_p),
        ("page_table", ctypes.c_void_p),
        ("x", ctypes.c_void_p),
        ("logits", ctypes.c_void_p),
        ("topk", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("mixer_out", ctypes.c_void_p),
        ("h_in", ctypes.c_void_p),
    ]


TOK_WORDS = 32  # sizeof(qres_tok) / 4: pos[8], token[8], feed, step, slot, reserved[13]
TOK_POS, TOK_TOKEN, TOK_FEED, TOK_STEP, TOK_SLOT = 0, 8, 16, 17, 18

_lib = None


def lib():
    """the loaded libqres.so (raises if it is missing: there is no fallback)"""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise QresError(f"{LIB_PATH} is missing: build it with `python -m tt_qwen_resident_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        vp, i32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t
        sig = {
            "qres_create": [ctypes.POINTER(Config), i32, i32, ctypes.POINTER(vp)],
            "qres_destroy": [vp],
            "qres_last_error": [vp, ctypes.c_char_p, sz],
            "qres_load_weights": [vp, i32, i32, ctypes.POINTER(Weight)],
            "qres_load_gdn_params": [vp, i32, vp, vp, vp, vp],
            "qres_load_attn_params": [vp, i32, vp, vp],
            "qres_bind_state": [vp, i32, ctypes.POINTER(LayerState)],
            "qres_load_gdn_state": [vp, i32, i32, vp, vp, i32, vp],
            "qres_dump_gdn_state": [vp, i32, i32, vp, vp],
            "qres_load_kv": [vp, i32, i32, vp, vp, i32, vp],
            "qres_dump_kv": [vp, i32, i32, vp, vp, i32, vp],
            "qres_bind_rope": [vp, vp, vp, i32],
            "qres_bind_io": [vp, ctypes.POINTER(Io)],
            "qres_bind_sampling": [vp, vp],
            "qres_workspace_size": [vp, ctypes.POINTER(sz)],
            "qres_bind_workspace": [vp, vp, sz],
            "qres_nccl_unique_id": [ctypes.c_char_p, vp],
            "qres_nccl_init": [vp, ctypes.c_char_p, vp],
            "qres_p2p_window_size": [vp, ctypes.POINTER(sz)],
            "qres_p2p_alloc": [vp, vp],
            "qres_p2p_open": [vp, vp],
            "qres_decode_step": [vp, vp],
            "qres_capture": [vp, vp],
            "qres_replay": [vp, vp],
            "qres_release_graph": [vp],
            "qres_check": [vp, vp],
            "qres_wait_probe": [vp, vp, ctypes.c_uint32, ctypes.c_uint32, vp],
            "qres_gemv_workspace_size": [i32, i32, ctypes.POINTER(sz)],
            "qres_gemv": [ctypes.POINTER(Weight), i32, i32, vp, i32, vp, i32, vp, vp, sz, vp],
            "qres_gdn_mixer": [i32, i32, vp, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp],
            "qres_attn_workspace_size": [i32, i32, i32, ctypes.POINTER(sz)],
            "qres_attn_mixer": [i32, i32, vp, i32, vp, vp, i32, vp, vp, vp, vp, vp, vp, vp, vp, sz, vp, vp],
            "qres_topk_workspace_size": [i32, i32, ctypes.POINTER(sz)],
            "qres_topk": [i32, vp, i32, i32, vp, vp, vp, sz, vp],
            "qres_topk_noalloc": [i32, vp, i32, i32, vp, vp, vp],
            "qres_sample": [i32, vp, vp, vp, vp, vp],
            "qres_quantize_fp8": [vp, i32, i32, vp, vp, vp],
            "qres_tile_weight": [vp, i32, i32, vp, vp],
        }
        for name, args in sig.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = ctypes.c_int
        for name in ("qres_step_launches", "qres_exchange_mode"):
            getattr(L, name).argtypes = [vp]
            getattr(L, name).restype = ctypes.c_int32
        _lib = L
    return _lib


def last_error(ctx=None):
    buf = ctypes.create_string_buffer(1024)
    lib().qres_last_error(ctx, buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status, ctx=None, what=""):
    if status != 0:
        raise QresError(f"{what}: {STATUS.get(status, status)}: {last_error(ctx)}")


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def stream_ptr(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


# ------------------------------------------------------------------------------ single-kernel ops (torch.ops.qres)
_gemv_work = {}


def gemv_work(device, rows_pad, grid=0):
    """a zeroed GEMV workspace for weights of up to rows_pad rows (cached per device)"""
    sz = ctypes.c_size_t()
    check(lib().qres_gemv_workspace_size(grid, rows_pad, ctypes.byref(sz)), None, "gemv ws")
    key = (str(device), grid)
    w = _gemv_work.get(key)
    if w is None or w.numel() < sz.value:
        w = torch.zeros(sz.value, dtype=torch.uint8, device=device)
        _gemv_work[key] = w
    return w


def gemv(w, h, pro, epi, out, err=None, grid=0, stream=None, work=None):
    """one weight-streaming projection (see qres_gemv); w a GemvWeight, h [rows][K] (fp32 x or bf16), out
    preallocated"""
    rows = h.shape[0]
    work = work if work is not None else gemv_work(h.device, w.rows_pad, grid)
    check(
        lib().qres_gemv(ctypes.byref(w.cstruct()), rows, pro, ptr(h), epi, ptr(out), grid, ptr(err), ptr(work),
                        work.numel(), stream_ptr(stream)),
        None,
        "qres_gemv",
    )
    return out


def quantize_fp8(w, stream=None):
    """fp32 [N][K] (device) -> (uint8 [N][K], fp32 scales [ceil(N/128)][ceil(K/128)]) on the GPU"""
    N, K = w.shape
    q = torch.empty(N, K, dtype=torch.uint8, device=w.device)
    s = torch.empty(-(-N // 128), -(-K // 128), dtype=torch.float32, device=w.device)
    check(lib().qres_quantize_fp8(ptr(w.contiguous()), N, K, ptr(q), ptr(s), stream_ptr(stream)), None, "quantize")
    return q, s


def tile_weight(q, stream=None):
    """row-major e4m3 [rows][K] (device) -> the GEMV layout (rows padded to a multiple of 128)"""
    rows, K = q.shape
    rows_pad = (rows + 127) // 128 * 128
    dst = torch.empty(rows_pad * K, dtype=torch.uint8, device=q.device)
    check(lib().qres_tile_weight(ptr(q.contiguous()), rows, K, ptr(dst), stream_ptr(stream)), None, "tile")
    return dst


def topk(logits, base=0, work=None, stream=None):
    """bf16 logits [rows][n] -> (lists uint32 [rows][64], argmax int32 [rows])"""
    rows, n = logits.shape
    sz = ctypes.c_size_t()
    check(lib().qres_topk_workspace_size(rows, n, ctypes.byref(sz)), None, "topk ws")
    if work is None:
        work = torch.zeros(sz.value, dtype=torch.uint8, device=logits.device)
    lists = torch.empty(rows, 2 * QRES_TOPK, dtype=torch.int32, device=logits.device)
    am = torch.empty(rows, dtype=torch.int32, device=logits.device)
    check(
        lib().qres_topk(rows, ptr(logits), n, base, ptr(lists), ptr(am), ptr(work), work.numel(), stream_ptr(stream)),
        None,
        "topk",
    )
    return lists, am
