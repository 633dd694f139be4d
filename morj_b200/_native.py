"""ctypes binding of the C-ABI library `_morj_b200.so` (declared in `include/morj_b200.h`).

The engine's only route to the GPU kernels. There is no fallback: if the library is missing or fails to load,
`lib()` raises, and every wrapper raises on a non-zero status (`ValueError` for bad arguments, `MemoryError` for
out-of-memory, `NativeFailure` otherwise), mirroring the reference engine's error classes.
"""
import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, '_morj_b200.so')

OK, ERR_ARG, ERR_CUDA, ERR_OOM, ERR_TIMEOUT, ERR_UNSUPPORTED, ERR_INTERNAL = 0, 1, 2, 3, 4, 5, 6
EPI_STORE, EPI_GEGLU = 0, 1

_lock = threading.Lock()
_lib = None

P = ctypes.c_void_p
I = ctypes.c_int
LL = ctypes.c_longlong
F = ctypes.c_float
IP = ctypes.POINTER(ctypes.c_int)

# name -> argument types (all return int, except morj_last_error)
SIGNATURES = {
    'morj_version': [],
    'morj_device_error': [IP, I, P],
    'morj_gemm_bf16': [P, LL, P, LL, P, LL, I, I, I, I, P],
    'morj_gemm_workspace_bytes': [ctypes.POINTER(ctypes.c_ulonglong)],
    'morj_gemm_workspace_set': [P, P, ctypes.c_ulonglong],
    'morj_gemm_workspace_remove': [P],
    'morj_gemm_split_walk': [I, I, I, I, IP, I],
    'morj_gemm_skinny_walk': [I, I, I, I, IP, I],
    'morj_gemm_qkv_rope': [P, LL, P, LL, I, I, I, I, I, I, P, P, P, P, I, P, F, P, P, P, P],
    'morj_rope_table': [P, I, I, P, P],
    'morj_embed_rmsnorm': [P, P, P, P, I, I, F, P, F, P, P, P],
    'morj_qkv_post': [P, LL, I, I, I, I, I, P, P, P, P, P, F, P, P, P, P],
    'morj_tree_attention_work': [IP, IP, IP, I, I, I, I, I, I, IP, I],
    'morj_tree_attention': [P, I, P, P, I, P, P, P, P, P, I, I, I, I, I, I, I, F, P, I, P],
    'morj_attn_epilogue': [P, P, P, P, P, I, I, F, P],
    'morj_mlp_epilogue': [P, P, P, P, P, P, I, I, F, I, P],
    'morj_gather_rows': [P, LL, P, I, I, P, LL, P],
    'morj_scatter_rows': [P, LL, P, I, I, P, LL, P],
    'morj_label_head': [P, LL, P, P, P, I, P, P, I, F, F, P, P],
    'morj_geglu': [P, I, I, P, P],
    'morj_ipc_export': [P, P],
    'morj_ipc_import': [P, ctypes.POINTER(P)],
    'morj_ipc_close': [P, P],
    'morj_gemm_bf16_peer': [P, LL, P, LL, I, I, I, P, P],
    'morj_peer_reduce': [P, I, I, P, P, P, F, I, I, ctypes.c_ulonglong, P],
    'morj_peer_wait': [P, I, ctypes.c_ulonglong, P],
    'morj_gemm_norm_epilogue_noalloc': [P, LL, P, LL, I, I, I, I, P, P, P, P, P, F, I, P],
    'morj_vision_patch_prologue': [P, LL, P],
    'morj_vision_position_add': [P, P, P, I, I, I, P],
    'morj_vision_head_epilogue': [P, LL, I, I, I, P, P, P, P, F, P, P, P, P],
    'morj_vision_pool': [P, I, P, P, I, F, F, P, P],
    'morj_rmsnorm_rows': [P, P, I, I, F, P, P],
    'morj_tree_build': [P, P, I, ctypes.POINTER(P)],
    'morj_tree_layout': [P, P, P, P, P, P, P, P],
    'morj_plan_pass': [P, P, I, P, I, I, LL, LL, I, P, LL, P, P, P, LL, P, LL, P, I, ctypes.POINTER(P)],
    'morj_plan_blob': [P, ctypes.POINTER(ctypes.POINTER(ctypes.c_longlong)), ctypes.POINTER(LL)],
}
VOID_SIGNATURES = {'morj_tree_free': [P], 'morj_plan_free': [P]}

IPC_HANDLE_BYTES = 72
MAX_RANKS = 8


class PeerDesc(ctypes.Structure):
    """`morj_peer_t`: the exchange buffers of every rank of a tensor-parallel group, as this process sees them."""
    _fields_ = [('world', I), ('rank', I), ('max_blocks', I), ('hidden', I),
                ('part', P * MAX_RANKS), ('x', P * MAX_RANKS), ('h', P * MAX_RANKS),
                ('partials', P * MAX_RANKS), ('rows', P * MAX_RANKS)]


class NativeFailure(RuntimeError):
    """A native call failed for a reason other than bad arguments or memory (the engine treats it as fatal)."""


def lib():
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(f'native library {LIB_PATH} is not built (python -m morj_b200.build)')
                L = ctypes.CDLL(LIB_PATH)
                for name, args in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.argtypes = args
                    fn.restype = ctypes.c_int
                for name, args in VOID_SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.argtypes = args
                    fn.restype = None
                L.morj_last_error.argtypes = []
                L.morj_last_error.restype = ctypes.c_char_p
                _lib = L
    return _lib


def check(status, what):
    if status == OK:
        return
    msg = lib().morj_last_error().decode(errors='replace')
    text = f'{what}: {msg}'
    if status == ERR_ARG:
        raise ValueError(text)
    if status == ERR_OOM:
        raise MemoryError(text)
    if status == ERR_INTERNAL:
        raise AssertionError(text)
    raise NativeFailure(f'{text} (status {status})')


def call(name, *args):
    """Call entry point `name` and raise on a non-zero status."""
    check(getattr(lib(), name)(*args), name)


def attention_work(qo_indptr, kv_indptr, n_bidir, hq, hk, window, page_size=1, kv_last_page_len=None):
    """The attention work list (int32 pairs, longest tiles first) for host copies of a call's segment tables."""
    import numpy as np
    qo = np.ascontiguousarray(qo_indptr, dtype=np.int32)
    kv = np.ascontiguousarray(kv_indptr, dtype=np.int32)
    last = None if kv_last_page_len is None else np.ascontiguousarray(kv_last_page_len, dtype=np.int32)
    n_seg = len(qo) - 1
    qt = 128 // (hq // hk)
    cap = max(1, int(sum((int(qo[i + 1] - qo[i]) + qt - 1) // qt for i in range(n_seg))))
    buf = np.zeros(2 * cap, dtype=np.int32)
    got = lib().morj_tree_attention_work(qo.ctypes.data_as(IP), kv.ctypes.data_as(IP),
                                         last.ctypes.data_as(IP) if last is not None else None, n_seg, n_bidir, hq, hk,
                                         page_size, window, buf.ctypes.data_as(IP), cap)
    if got < 0:
        check(ERR_ARG, 'morj_tree_attention_work')
    return buf[:2 * got]


def device_error(stream, clear=True):
    """The device error word (0 = no kernel reported a failure); synchronises `stream`."""
    code = ctypes.c_int(0)
    check(lib().morj_device_error(ctypes.byref(code), int(clear), stream), 'morj_device_error')
    return code.value


def gemm_workspace_bytes():
    """Bytes of a split-tile workspace for the pair GEMM kernel on the current device."""
    n = ctypes.c_ulonglong(0)
    check(lib().morj_gemm_workspace_bytes(ctypes.byref(n)), 'morj_gemm_workspace_bytes')
    return n.value


def split_walk(tiles, pairs, kblocks, pair):
    """The pair GEMM kernel's work items for SM pair `pair`, in order: an [n, 4] int32 array of
    (tile, first k-block, end k-block, kind) with kind 0 whole, 1 head of a cut tile, 2 tail of a cut tile."""
    import numpy as np
    cap = tiles // max(1, pairs) + 4
    buf = np.zeros(4 * cap, dtype=np.int32)
    n = lib().morj_gemm_split_walk(tiles, pairs, kblocks, pair, buf.ctypes.data_as(IP), cap)
    if n < 0:
        check(ERR_ARG, 'morj_gemm_split_walk')
    return buf[:4 * n].reshape(n, 4)


def skinny_walk(tiles, kblocks, ctas, cta):
    """The weight-streaming kernel's work for CTA `cta` of `ctas`: an [n, 5] int32 array of (tile, first k-block,
    end k-block, piece, pieces)."""
    import numpy as np
    cap = tiles * kblocks // ctas + 3
    buf = np.zeros(5 * cap, dtype=np.int32)
    n = lib().morj_gemm_skinny_walk(tiles, kblocks, ctas, cta, buf.ctypes.data_as(IP), cap)
    if n < 0:
        check(ERR_ARG, 'morj_gemm_skinny_walk')
    return buf[:5 * n].reshape(n, 5)


class GemmWorkspace:
    """Device memory for the pair GEMM kernel's split tiles, registered (`morj_gemm_workspace_set`) for each stream it
    serves; `close()` (or garbage collection) unregisters it before the memory goes back to torch."""

    def __init__(self, device):
        import torch
        self.nbytes = gemm_workspace_bytes()
        self.buf = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        self.ptr = self.buf.data_ptr()
        self.streams = set()

    def register(self, stream):
        if self.ptr and stream not in self.streams:
            call('morj_gemm_workspace_set', stream, self.ptr, self.nbytes)
            self.streams.add(stream)

    def close(self):
        if self.ptr:
            lib().morj_gemm_workspace_remove(self.ptr)
            self.ptr = None
            self.streams.clear()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
