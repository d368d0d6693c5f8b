"""eakv_b200 - Python host binding of libeakv_b200.so.

The library is the product: a C-ABI shared library (include/eakv.h,
include/eakv_cuda.h) whose kernels are hand-written sm_100a CUDA. This module
is a thin ctypes layer over it that mirrors the reference's C API one for one
(petlukk/eakv include/eakv.h:25-83: same function names, same argument
meaning, same integer return codes), plus a small `Cache` convenience class.
There is no CPU implementation behind any of these calls: if the shared
library is missing or cannot be loaded, importing `lib()` raises.

Array arguments accept numpy float32 arrays (host pointers) or any object
exposing `data_ptr()` (torch CUDA tensors, device pointers) for the *_device
entry points.
"""
import ctypes
import os

import numpy as np

EAKV_OK = 0
EAKV_ERR_IO = -1
EAKV_ERR_FORMAT = -2
EAKV_ERR_ALLOC = -3
EAKV_ERR_INVALID = -4

_HERE = os.path.dirname(os.path.abspath(__file__))
# EAKV_B200_LIB selects another build of the library (same ABI)
LIB_PATH = os.environ.get("EAKV_B200_LIB") or os.path.join(_HERE, "libeakv_b200.so")

_c = ctypes
_P = _c.c_void_p
_I = _c.c_int
_F = _c.c_float

# name -> (restype, argtypes); every symbol declared in the headers of
# include/.
SIGNATURES = {
    # eakv.h
    "eakv_cache_create": (_P, [_I, _I, _I, _I]),
    "eakv_cache_free": (None, [_P]),
    "eakv_cache_load_raw": (_I, [_P, _P, _I]),
    "eakv_cache_append": (_I, [_P, _P, _I, _I, _I]),
    "eakv_cache_advance": (_I, [_P, _I]),
    "eakv_cache_clear": (None, [_P]),
    "eakv_checkpoint": (_I, [_P]),
    "eakv_restore": (_I, [_P, _I]),
    "eakv_attention_scores": (None, [_P, _P, _I, _I, _I, _P]),
    "eakv_attention_output": (None, [_P, _P, _I, _I, _I, _P]),
    "eakv_cache_save": (_I, [_P, _c.c_char_p]),
    "eakv_cache_load": (_I, [_c.c_char_p, _c.POINTER(_P)]),
    "eakv_cache_seq_len": (_I, [_P]),
    "eakv_cache_n_layers": (_I, [_P]),
    "eakv_cache_n_heads": (_I, [_P]),
    "eakv_cache_head_dim": (_I, [_P]),
    "eakv_cache_max_seq_len": (_I, [_P]),
    "eakv_cache_compression_ratio": (_F, [_P]),
    # eakv_cuda.h
    "eakv_last_error": (_I, []),
    "eakv_last_error_string": (_c.c_char_p, []),
    "eakv_device_status": (_I, [_I, _I]),
    "eakv_set_device": (_I, [_I]),
    "eakv_cache_device": (_I, [_P]),
    "eakv_cache_device_bytes": (_c.c_size_t, [_P]),
    "eakv_cache_set_stream": (_I, [_P, _P]),
    "eakv_cache_stream": (_P, [_P]),
    "eakv_cache_synchronize": (_I, [_P]),
    "eakv_cache_load_raw_device": (_I, [_P, _P, _I]),
    "eakv_cache_append_device": (_I, [_P, _P, _I, _I, _I]),
    "eakv_cache_append_step_device": (_I, [_P, _P, _I]),
    "eakv_attention_scores_device": (_I, [_P, _P, _I, _I, _I, _P]),
    "eakv_attention_output_device": (_I, [_P, _P, _I, _I, _I, _P]),
    "eakv_attention_fused": (_I, [_P, _P, _I, _I, _I, _P]),
    "eakv_attention_fused_device": (_I, [_P, _P, _I, _I, _I, _P]),
    "eakv_decode_attention": (_I, [_P, _I, _P, _I, _P, _P]),
    "eakv_decode_attention_host": (_I, [_P, _I, _P, _I, _P, _P]),
    "eakv_decode_attention_noalloc": (_I, [_P, _I, _P, _I, _P, _P]),
    "eakv_decode_launches": (_I, [_P, _I, _I]),
    "eakv_decode_splits": (_I, [_P, _I, _I]),
    "eakv_decode_attention_partial": (_I, [_P, _I, _P, _I, _I, _I, _P, _P, _P]),
    "eakv_lse_combine": (_I, [_I, _I, _I, _P, _P, _P, _P, _P]),
    "eakv_test_force_splits": (_I, [_I]),
    "eakv_test_force_path": (_I, [_I]),
    "eakv_test_choose_splits": (_I, [_c.c_longlong, _I, _I, _I, _I, _I]),
    "eakv_test_stall": (_I, [_I, ctypes.c_uint]),
    "eakv_test_separate_merge": (_I, [_I]),
    "eakv_cache_validate": (_I, [_P, _P]),
    "eakv_cache_dequantize_device": (_I, [_P, _I, _I, _I, _I, _P, _P]),
    "eakv_cache_dequantize": (_I, [_P, _I, _I, _I, _I, _P]),
    # eakv_nccl.h
    "eakv_nccl_version": (_I, []),
    "eakv_nccl_unique_id": (_I, [_P]),
    "eakv_nccl_comm_init": (_I, [_c.POINTER(_P), _I, _P, _I, _I]),
    "eakv_nccl_comm_destroy": (_I, [_P]),
    "eakv_nccl_comm_abort": (_I, [_P]),
    "eakv_decode_attention_split": (_I, [_P, _I, _P, _I, _I, _I, _P, _P, _P]),
    "eakv_decode_attention_split_host": (_I, [_P, _I, _P, _I, _P, _P, _P]),
    # eakv_ggml.h
    "eakv_quantize_row": (None, [_P, _P, _c.c_int64]),
    "eakv_dequantize_row": (None, [_P, _P, _c.c_int64]),
    "eakv_vec_dot_q4_f32": (None, [_I, _P, _c.c_size_t, _P, _c.c_size_t, _P, _c.c_size_t, _I]),
    # eakv_llama.h
    "eakv_from_llama_state": (_I, [_P, _c.c_size_t, _I, _I, _I, _I, _c.POINTER(_P)]),
    "eakv_from_llama_state_append": (_I, [_P, _P, _c.c_size_t, _I, _I, _I, _I]),
    "eakv_ggml_quantize_row_device": (_I, [_P, _P, _c.c_int64, _P]),
    "eakv_ggml_dequantize_row_device": (_I, [_P, _P, _c.c_int64, _P]),
    "eakv_ggml_vec_dot_device": (_I, [_I, _P, _c.c_size_t, _P, _c.c_size_t, _P, _c.c_size_t, _I,
                                      _P]),
}

_lib = None


def lib():
    """The loaded libeakv_b200.so (raises if it is absent: no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing; build it with `python -m eakv_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error():
    L = lib()
    return L.eakv_last_error(), (L.eakv_last_error_string() or b"").decode()


class EakvError(RuntimeError):
    def __init__(self, rc, what):
        code, msg = last_error()
        super().__init__(f"{what} failed: rc={rc} ({msg})")
        self.rc = rc


def _ptr(x):
    """Pointer of a numpy array (host) or of an object with data_ptr()."""
    if x is None:
        return None
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if isinstance(x, int):
        return x
    raise TypeError(f"cannot take a pointer of {type(x)}")


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a


def _check(rc, what):
    if rc != EAKV_OK:
        raise EakvError(rc, what)
    return rc


class Cache:
    """Owning wrapper of one eakv_cache_t (device-resident Q4 cache)."""

    def __init__(self, n_layers=None, n_kv_heads=None, head_dim=None, max_seq_len=None,
                 _handle=None):
        L = lib()
        if _handle is not None:
            self.h = _handle
        else:
            self.h = L.eakv_cache_create(n_layers, n_kv_heads, head_dim, max_seq_len)
            if not self.h:
                raise EakvError(None, "eakv_cache_create")

    # --- lifecycle ---------------------------------------------------------
    def free(self):
        if self.h:
            lib().eakv_cache_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.free()

    @classmethod
    def load(cls, path):
        out = ctypes.c_void_p()
        _check(lib().eakv_cache_load(os.fsencode(path), ctypes.byref(out)), "eakv_cache_load")
        return cls(_handle=out.value)

    @classmethod
    def from_llama_state(cls, state, n_layers, n_kv_heads, head_dim, max_seq_len):
        """eakv_from_llama_state on a host bytes object (a llama.cpp
        sequence state); raises EakvError with the reference's code."""
        buf = np.frombuffer(state, np.uint8)
        out = ctypes.c_void_p()
        _check(lib().eakv_from_llama_state(_ptr(buf), buf.size, n_layers, n_kv_heads, head_dim,
                                           max_seq_len, ctypes.byref(out)),
               "eakv_from_llama_state")
        return cls(_handle=out.value)

    def append_llama_state(self, state, n_layers, n_kv_heads, head_dim, start_pos):
        """eakv_from_llama_state_append; returns the reference's code."""
        buf = np.frombuffer(state, np.uint8)
        return lib().eakv_from_llama_state_append(self.h, _ptr(buf), buf.size, n_layers,
                                                  n_kv_heads, head_dim, start_pos)

    # --- inspection ----------------------------------------------------------------
    def validate(self):
        """eakv_cache_validate: int32[n_layers*2] codes (0 ok, 1 NaN scale,
        2 NaN bias, 3 negative scale), index layer*2 + kv."""
        codes = np.zeros(self.n_layers * 2, np.int32)
        _check(lib().eakv_cache_validate(self.h, _ptr(codes)), "eakv_cache_validate")
        return codes

    def dequantize(self, layer, kv_idx, pos_begin, pos_end):
        """f32[n_kv_heads][pos_end - pos_begin][head_dim] on the host."""
        out = np.zeros((self.n_kv_heads, max(pos_end - pos_begin, 0), self.head_dim), np.float32)
        _check(lib().eakv_cache_dequantize(self.h, layer, kv_idx, pos_begin, pos_end, _ptr(out)),
               "eakv_cache_dequantize")
        return out

    def dequantize_device(self, layer, kv_idx, pos_begin, pos_end, d_out, stream=None):
        return _check(lib().eakv_cache_dequantize_device(self.h, layer, kv_idx, pos_begin,
                                                         pos_end, _ptr(d_out), stream),
                      "eakv_cache_dequantize_device")

    # --- info ----------------------------------------------------------------
    @property
    def seq_len(self):
        return lib().eakv_cache_seq_len(self.h)

    @property
    def n_layers(self):
        return lib().eakv_cache_n_layers(self.h)

    @property
    def n_kv_heads(self):
        return lib().eakv_cache_n_heads(self.h)

    @property
    def head_dim(self):
        return lib().eakv_cache_head_dim(self.h)

    @property
    def max_seq_len(self):
        return lib().eakv_cache_max_seq_len(self.h)

    @property
    def device(self):
        return lib().eakv_cache_device(self.h)

    @property
    def device_bytes(self):
        return lib().eakv_cache_device_bytes(self.h)

    def compression_ratio(self):
        return lib().eakv_cache_compression_ratio(self.h)

    # --- quantize --------------------------------------------------------------
    def load_raw(self, data, seq_len):
        data = _f32(data)
        return lib().eakv_cache_load_raw(self.h, _ptr(data), seq_len)

    def append(self, data, layer, kv_idx, n_tokens):
        data = _f32(data)
        return lib().eakv_cache_append(self.h, _ptr(data), layer, kv_idx, n_tokens)

    def advance(self, n):
        return lib().eakv_cache_advance(self.h, n)

    def clear(self):
        lib().eakv_cache_clear(self.h)

    def checkpoint(self):
        return lib().eakv_checkpoint(self.h)

    def restore(self, seq_len):
        return lib().eakv_restore(self.h, seq_len)

    def save(self, path):
        return lib().eakv_cache_save(self.h, os.fsencode(path))

    # --- attention (host buffers, reference contract) -------------------------
    def scores(self, queries, layer, n_q, n_kv):
        q = _f32(queries)
        out = np.empty(n_q * self.seq_len, np.float32)
        lib().eakv_attention_scores(self.h, _ptr(q), layer, n_q, n_kv, _ptr(out))
        return out

    def output(self, weights, layer, n_q, n_kv):
        w = _f32(weights)
        out = np.empty(n_q * self.head_dim, np.float32)
        lib().eakv_attention_output(self.h, _ptr(w), layer, n_q, n_kv, _ptr(out))
        return out

    def fused(self, queries, layer, n_q, n_kv):
        q = _f32(queries)
        out = np.empty(n_q * self.head_dim, np.float32)
        _check(lib().eakv_attention_fused(self.h, _ptr(q), layer, n_q, n_kv, _ptr(out)),
               "eakv_attention_fused")
        return out

    # --- device entry points ------------------------------------------------------
    def scores_device(self, d_queries, layer, n_q, n_kv, d_scores):
        """eakv_attention_scores_device: f32[n_q][seq_len] scores on the device."""
        return _check(lib().eakv_attention_scores_device(self.h, _ptr(d_queries), layer, n_q, n_kv,
                                                         _ptr(d_scores)),
                      "eakv_attention_scores_device")

    def output_device(self, d_weights, layer, n_q, n_kv, d_output):
        """eakv_attention_output_device: f32[n_q][head_dim] outputs on the device."""
        return _check(lib().eakv_attention_output_device(self.h, _ptr(d_weights), layer, n_q, n_kv,
                                                         _ptr(d_output)),
                      "eakv_attention_output_device")

    def load_raw_device(self, d_data, seq_len):
        return lib().eakv_cache_load_raw_device(self.h, _ptr(d_data), seq_len)

    def append_device(self, d_data, layer, kv_idx, n_tokens):
        return lib().eakv_cache_append_device(self.h, _ptr(d_data), layer, kv_idx, n_tokens)

    def append_step_device(self, d_data, n_tokens):
        return lib().eakv_cache_append_step_device(self.h, _ptr(d_data), n_tokens)

    def set_stream(self, stream_handle):
        return _check(lib().eakv_cache_set_stream(self.h, stream_handle), "set_stream")

    def synchronize(self):
        return _check(lib().eakv_cache_synchronize(self.h), "synchronize")


def _handles(caches):
    arr = (ctypes.c_void_p * len(caches))(*[c.h for c in caches])
    return arr


def decode_attention(caches, d_queries, n_q_heads, d_output, stream=None):
    """Batched fused decode over device buffers (see eakv_cuda.h)."""
    arr = _handles(caches)
    return _check(lib().eakv_decode_attention(arr, len(caches), _ptr(d_queries), n_q_heads,
                                              _ptr(d_output), stream),
                  "eakv_decode_attention")


def decode_attention_noalloc(caches, d_queries, n_q_heads, d_output, stream=None):
    """eakv_decode_attention without any device allocation (fixed 4 MiB
    workspace in the library; see eakv_cuda.h). Returns the C return code."""
    arr = _handles(caches)
    return lib().eakv_decode_attention_noalloc(arr, len(caches), _ptr(d_queries), n_q_heads,
                                               _ptr(d_output), stream)


def decode_attention_host(caches, queries, n_q_heads, output, stream=None):
    arr = _handles(caches)
    return _check(lib().eakv_decode_attention_host(arr, len(caches), _ptr(queries), n_q_heads,
                                                   _ptr(output), stream),
                  "eakv_decode_attention_host")


def decode_attention_partial(caches, d_queries, n_q_heads, pos_begin, pos_end, d_output,
                             d_lse, stream=None):
    arr = _handles(caches)
    return _check(lib().eakv_decode_attention_partial(arr, len(caches), _ptr(d_queries),
                                                      n_q_heads, pos_begin, pos_end,
                                                      _ptr(d_output), _ptr(d_lse), stream),
                  "eakv_decode_attention_partial")


def lse_combine(n_parts, n_rows, head_dim, d_parts, d_lse, d_output, d_lse_out=None,
                stream=None):
    return _check(lib().eakv_lse_combine(n_parts, n_rows, head_dim, _ptr(d_parts), _ptr(d_lse),
                                         _ptr(d_output), _ptr(d_lse_out), stream),
                  "eakv_lse_combine")


# --- sequence split over NCCL (include/eakv_nccl.h) -------------------------------
NCCL_ID_BYTES = 128


def nccl_version():
    """NCCL version code of the library's NCCL (< 0: unavailable)."""
    return lib().eakv_nccl_version()


def nccl_unique_id():
    """A new NCCL unique id (bytes) for eakv_nccl_comm_init."""
    buf = ctypes.create_string_buffer(NCCL_ID_BYTES)
    _check(lib().eakv_nccl_unique_id(buf), "eakv_nccl_unique_id")
    return buf.raw


class NcclComm:
    """A communicator of the library's NCCL (eakv_nccl_comm_init): n_ranks
    ranks, this one `rank`, on CUDA device `device`; blocks until every rank
    has joined."""

    def __init__(self, n_ranks, unique_id, rank, device):
        if len(unique_id) != NCCL_ID_BYTES:
            raise ValueError("bad NCCL unique id")
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(unique_id), NCCL_ID_BYTES)
        _check(lib().eakv_nccl_comm_init(ctypes.byref(h), n_ranks, buf, rank, device),
               "eakv_nccl_comm_init")
        self.h = h.value
        self.n_ranks, self.rank, self.device = n_ranks, rank, device

    def destroy(self):
        if self.h:
            _check(lib().eakv_nccl_comm_destroy(self.h), "eakv_nccl_comm_destroy")
            self.h = None

    def abort(self):
        if self.h:
            lib().eakv_nccl_comm_abort(self.h)
            self.h = None


def decode_attention_split(caches, d_queries, n_q_heads, d_output, comm, pos_begin=0,
                           pos_end=-1, stream=None):
    """eakv_decode_attention_split: this rank's slice of every sequence,
    merged with the other ranks' over `comm` (an NcclComm)."""
    arr = _handles(caches)
    return _check(lib().eakv_decode_attention_split(arr, len(caches), _ptr(d_queries), n_q_heads,
                                                    pos_begin, pos_end, _ptr(d_output), comm.h,
                                                    stream),
                  "eakv_decode_attention_split")


def decode_attention_split_host(caches, queries, n_q_heads, output, comm, stream=None):
    """eakv_decode_attention_split_host: host queries in, merged host output
    out, copies overlapped with the chunks' split steps."""
    arr = _handles(caches)
    return _check(lib().eakv_decode_attention_split_host(arr, len(caches), _ptr(queries),
                                                         n_q_heads, _ptr(output), comm.h, stream),
                  "eakv_decode_attention_split_host")


def decode_launches(caches, n_q_heads):
    return lib().eakv_decode_launches(_handles(caches), len(caches), n_q_heads)


def decode_splits(caches, n_q_heads):
    """Sequence splits per row the planner picks for these caches."""
    return lib().eakv_decode_splits(_handles(caches), len(caches), n_q_heads)


def set_device(device):
    """Selects the device for caches created later on this thread."""
    return _check(lib().eakv_set_device(int(device)), "eakv_set_device")


def device_status(device=0, reset=False):
    return lib().eakv_device_status(device, 1 if reset else 0)


def force_splits(n):
    lib().eakv_test_force_splits(int(n))


def choose_splits(items, max_pages, lo, hi, per_sm, sms):
    """The decode planner's split count for `items` rows of max_pages pages,
    searched in [lo, hi], with per_sm CTAs resident on each of `sms` SMs
    (host code only: runs without a GPU)."""
    return lib().eakv_test_choose_splits(int(items), int(max_pages), int(lo), int(hi),
                                         int(per_sm), int(sms))


def separate_merge(on):
    """Test aid: merge sequence splits in a second kernel (True) instead of
    inside the decode kernel (False, the default)."""
    lib().eakv_test_separate_merge(1 if on else 0)


def force_path(path):
    """Decode kernel of later calls on this thread: 1 the CUDA-core kernel, 2 the
    mma.sync tensor-core kernel, 3 the tcgen05 tensor-core kernel (head_dim
    128), 0 the automatic choice."""
    lib().eakv_test_force_path(int(path))


def test_stall(page, wait_budget=0):
    """Failure-detection aid: decode kernels never request `page` of a work
    item (page < 0: off) and give up each wait after `wait_budget` polls."""
    lib().eakv_test_stall(int(page), int(wait_budget))


# --- q4_1_eakv ggml block type on device buffers (include/eakv_ggml.h) ------------
def ggml_quantize_row_device(d_src, d_dst, k, stream=None):
    return _check(lib().eakv_ggml_quantize_row_device(_ptr(d_src), _ptr(d_dst), int(k),
                                                      stream), "ggml_quantize_row_device")


def ggml_dequantize_row_device(d_src, d_dst, k, stream=None):
    return _check(lib().eakv_ggml_dequantize_row_device(_ptr(d_src), _ptr(d_dst), int(k),
                                                        stream), "ggml_dequantize_row_device")


def ggml_vec_dot_device(n, d_s, bs, d_vx, bx, d_vy, by, nrc, stream=None):
    return _check(lib().eakv_ggml_vec_dot_device(int(n), _ptr(d_s), bs, _ptr(d_vx), bx,
                                                 _ptr(d_vy), by, int(nrc), stream),
                  "ggml_vec_dot_device")
