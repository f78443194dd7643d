"""B200 (sm_100a) decode-attention backend for tmac_gguf.cpp -- Python host API.

A thin ctypes layer over ``libtg_cuda_backend.so`` (C ABI:
include/tg_cuda_backend.h).  ``CudaBackend`` mirrors the reference's
``metal_backend`` operator surface for this path -- ``init`` / ``shutdown``
(metal_backend.cpp:21-89), ``metal_batch_begin`` / ``metal_batch_end``
(metal_backend.hpp:114-191), ``rope_op`` (:381), ``elem_op`` (:354) and
``attention_op`` (:413) -- with the same argument order and meaning, so code
written against the reference's dispatch helpers reads the same here.
``KVCache`` adds the B200-native surface: device-resident caches, batched
variable-length decode, bf16 caches and split-KV decode across GPUs.

Arrays may be numpy arrays (host memory; staged by the library), torch CUDA
tensors, or raw integer device addresses.  There is no CPU fallback: every
op runs the CUDA kernels, and importing this module on a machine without
the built library raises.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import Optional

import numpy as np

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libtg_cuda_backend.so")
HEADER_PATH = os.path.join(PKG_DIR, "..", "include", "tg_cuda_backend.h")

TG_OK = 0
TG_ERR_INVALID_ARG = 1
TG_ERR_CUDA = 2
TG_ERR_NO_DEVICE = 3
TG_ERR_OUT_OF_MEMORY = 4
TG_ERR_UNSUPPORTED = 5
TG_ERR_DEVICE = 6
TG_ERR_COMM = 7
TG_ERR_STATE = 8

DTYPE_F32 = 0
DTYPE_BF16 = 1
WTYPE_Q5_0, WTYPE_Q8_0 = 6, 8  # GGML block types (TG_WTYPE_*)
PROFILE_ATTENTION, PROFILE_PROJECTION, PROFILE_STAMPS = 1, 2, 4  # tg_profile_enable masks

# split-KV record exchange (tg_comm_set_exchange)
EXCHANGE_AUTO, EXCHANGE_PEER, EXCHANGE_NCCL = 0, 1, 2
REGION_MIRROR = 0
REGION_DEVICE_OWNED = 1

# Qwen2-0.5B attention shape and RoPE base (tmac_gguf.cpp:163-172, :991).
N_HEAD, N_KV_HEAD, HEAD_DIM, ROPE_BASE = 14, 2, 64, 1000000.0


class TGError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status
        self.message = message


def build() -> None:
    """Compile libtg_cuda_backend.so for sm_100a in this directory."""
    subprocess.run(["make", "-s", "-C", PKG_DIR, "all"], check=True)


class tg_kv_desc(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("n_seqs", C.c_int),
                ("max_ctx", C.c_int), ("n_head", C.c_int),
                ("n_kv_head", C.c_int), ("head_dim", C.c_int),
                ("dtype", C.c_int), ("shard_start", C.c_int),
                ("global_ctx", C.c_int), ("rope_base", C.c_float)]


class tg_qkv_weights(C.Structure):
    _fields_ = [("q_type", C.c_int), ("k_type", C.c_int), ("v_type", C.c_int),
                ("cols", C.c_int), ("w_q", C.c_void_p), ("w_k", C.c_void_p),
                ("w_v", C.c_void_p), ("b_q", C.c_void_p), ("b_k", C.c_void_p),
                ("b_v", C.c_void_p)]


class tg_tensor_info(C.Structure):
    _fields_ = [("name", C.c_char_p), ("rows", C.c_uint64), ("cols", C.c_uint64),
                ("n_bytes", C.c_uint64), ("type", C.c_uint32), ("data", C.c_void_p)]


_vp = C.c_void_p
_SIGS = {
    "tg_status_string": (C.c_char_p, [C.c_int]),
    "tg_last_error": (C.c_char_p, []),
    "tg_version": (C.c_char_p, []),
    "tg_init": (C.c_int, [C.c_int, C.POINTER(_vp)]),
    "tg_shutdown": (C.c_int, [_vp]),
    "tg_set_stream": (C.c_int, [_vp, _vp]),
    "tg_get_stream": (C.c_int, [_vp, C.POINTER(_vp)]),
    "tg_device_sms": (C.c_int, [_vp, C.POINTER(C.c_int)]),
    "tg_batch_begin": (C.c_int, [_vp]),
    "tg_batch_end": (C.c_int, [_vp]),
    "tg_synchronize": (C.c_int, [_vp]),
    "tg_register_host": (C.c_int, [_vp, _vp, C.c_size_t, C.c_int]),
    "tg_unregister_host": (C.c_int, [_vp, _vp]),
    "tg_region_sync": (C.c_int, [_vp, _vp, C.c_size_t, C.c_int]),
    "tg_rope_op": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.c_int, C.c_float]),
    "tg_elem_op": (C.c_int, [_vp, C.c_int, _vp, _vp, C.c_int]),
    "tg_attention_op": (C.c_int, [_vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int,
                                  C.c_int, C.c_int]),
    "tg_kv_create": (C.c_int, [_vp, C.POINTER(tg_kv_desc), C.POINTER(_vp)]),
    "tg_kv_destroy": (C.c_int, [_vp]),
    "tg_kv_reset": (C.c_int, [_vp]),
    "tg_kv_layer_ptrs": (C.c_int, [_vp, C.c_int, C.POINTER(_vp), C.POINTER(_vp)]),
    "tg_kv_fill_normal": (C.c_int, [_vp, C.c_uint64]),
    "tg_kv_write_rows": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                   _vp, _vp]),
    "tg_kv_read_rows": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                  _vp, _vp]),
    "tg_rope_cache_write": (C.c_int, [_vp, _vp, C.c_int, C.c_int, _vp, _vp,
                                      _vp, _vp]),
    "tg_attention_batched": (C.c_int, [_vp, _vp, C.c_int, C.c_int, _vp, _vp,
                                       _vp]),
    "tg_decode_layer": (C.c_int, [_vp, _vp, C.c_int, C.c_int, _vp, _vp, _vp,
                                  _vp, _vp]),
    "tg_comm_unique_id": (C.c_int, [_vp, C.c_size_t]),
    "tg_comm_init": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.c_int]),
    "tg_comm_destroy": (C.c_int, [_vp]),
    "tg_attention_splitkv": (C.c_int, [_vp, _vp, C.c_int, C.c_int, _vp, _vp,
                                       _vp]),
    "tg_decode_layer_splitkv": (C.c_int, [_vp, _vp, C.c_int, C.c_int, _vp,
                                          _vp, _vp, _vp, _vp]),
    "tg_prefill_layer": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.c_int, _vp, _vp,
                                   _vp, _vp]),
    "tg_attention_records": (C.c_int, [_vp, _vp, C.c_int, C.c_int, _vp, _vp,
                                       _vp]),
    "tg_merge_records": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                   _vp, _vp]),
    "tg_graph_begin": (C.c_int, [_vp]),
    "tg_graph_end": (C.c_int, [_vp, C.POINTER(_vp)]),
    "tg_graph_launch": (C.c_int, [_vp, _vp]),
    "tg_graph_destroy": (C.c_int, [_vp]),
    "tg_attention_noalloc": (C.c_int, [_vp, _vp, _vp, _vp, C.c_int, C.c_int,
                                       C.c_int, C.c_int, C.c_int, C.c_int,
                                       _vp, _vp, _vp]),
    "tg_launch_count": (C.c_int, [_vp, C.POINTER(C.c_longlong)]),
    "tg_profile_enable": (C.c_int, [_vp, C.c_int]),
    "tg_profile_read": (C.c_int, [_vp, C.POINTER(C.c_double),
                                  C.POINTER(C.c_longlong)]),
    "tg_comm_set_exchange": (C.c_int, [_vp, C.c_int]),
    "tg_comm_exchange": (C.c_int, [_vp, C.POINTER(C.c_int)]),
    "tg_kv_uses_tensor_cores": (C.c_int, [_vp, C.POINTER(C.c_int)]),
    "tg_fused_qkv_op": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, C.c_int,
                                  C.c_int, C.c_int, C.c_int, C.c_int]),
    "tg_matmul_q": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp]),
    "tg_qkv_rope_cache_write": (C.c_int, [_vp, _vp, C.c_int, C.c_int,
                                          C.POINTER(tg_qkv_weights), _vp, _vp, _vp]),
    "tg_decode_layer_x": (C.c_int, [_vp, _vp, C.c_int, C.c_int,
                                    C.POINTER(tg_qkv_weights), _vp, _vp, _vp]),
    "tg_decode_layer_splitkv_x": (C.c_int, [_vp, _vp, C.c_int, C.c_int,
                                            C.POINTER(tg_qkv_weights), _vp, _vp, _vp]),
    "tg_attn_output": (C.c_int, [_vp, C.c_int, C.c_int, _vp, C.c_int, C.c_int, _vp, _vp]),
    "tg_set_projection_split": (C.c_int, [C.c_int]),
    "tg_set_decode_tuning": (C.c_int, [C.c_int, C.c_int]),
    "tg_comm_set_wait_limit_ms": (C.c_int, [_vp, C.c_int]),
    "tg_profile_read_stamps": (C.c_int, [_vp, _vp, C.c_size_t, C.POINTER(C.c_int),
                                         C.POINTER(C.c_int)]),
    "tg_model_load_tmac": (C.c_int, [_vp, C.c_char_p, C.POINTER(_vp)]),
    "tg_model_destroy": (C.c_int, [_vp]),
    "tg_model_count": (C.c_int, [_vp, C.POINTER(C.c_int)]),
    "tg_model_tensor_at": (C.c_int, [_vp, C.c_int, C.POINTER(tg_tensor_info)]),
    "tg_model_find": (C.c_int, [_vp, C.c_char_p, C.POINTER(tg_tensor_info)]),
    "tg_model_read": (C.c_int, [_vp, C.c_int, _vp, C.c_size_t]),
    "tg_model_layer_attention": (C.c_int, [_vp, C.c_int, C.POINTER(tg_qkv_weights),
                                           C.POINTER(_vp), C.POINTER(C.c_int)]),
    "tg_attention_block": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.POINTER(tg_qkv_weights),
                                     C.c_int, _vp, _vp, _vp, _vp]),
    "tg_attention_block_splitkv": (C.c_int, [_vp, _vp, C.c_int, C.c_int,
                                             C.POINTER(tg_qkv_weights), C.c_int, _vp, _vp,
                                             _vp, _vp]),
}

_lib: Optional[C.CDLL] = None


def lib() -> C.CDLL:
    """Load libtg_cuda_backend.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing; build it with `make -C {PKG_DIR}` "
                "(there is no CPU fallback for this backend)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list:
    return sorted(_SIGS)


def _check(status: int) -> None:
    if status != TG_OK:
        msg = lib().tg_last_error().decode(errors="replace")
        raise TGError(status, msg)


def _ptr(x) -> Optional[int]:
    """Address of a numpy array, a torch tensor, or an int (None for None)."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("arrays must be C-contiguous")
        return x.ctypes.data
    if hasattr(x, "data_ptr"):
        if hasattr(x, "is_contiguous") and not x.is_contiguous():
            raise ValueError("tensors must be contiguous")
        return x.data_ptr()
    raise TypeError(f"cannot take the address of {type(x).__name__}")


def set_projection_split(split: int) -> None:
    """Cluster width of the tensor-core projections (tg_set_projection_split):
    1 to 8 CTAs splitting the columns, or 0 for the automatic choice."""
    _check(lib().tg_set_projection_split(int(split)))


def set_decode_tuning(ring_kb: int = 0, preload: int = 0) -> None:
    """Tuning of the bf16 decode kernel (tg_set_decode_tuning): K/V ring per
    CTA (0 automatic, 128 or 192 KB) and whether tiles may be loaded before
    the grid-dependency wait when that is safe."""
    _check(lib().tg_set_decode_tuning(int(ring_kb), int(preload)))


def shard_range(global_ctx: int, world: int, rank: int):
    """Global positions [start, start+length) held by `rank` when a context
    of global_ctx positions is split evenly over `world` GPUs (the last
    shard may be shorter)."""
    per = -(-global_ctx // world)
    start = min(rank * per, global_ctx)
    return start, max(0, min(per, global_ctx - start))


NOALLOC_MAX_SEQS = 4096


def attention_noalloc(stream: int, q, k_cache, v_cache, dtype: int, n_seqs: int,
                      max_ctx: int, past_len, out, device_status=None,
                      n_head: int = N_HEAD, n_kv_head: int = N_KV_HEAD,
                      head_dim: int = HEAD_DIM) -> None:
    """tg_attention_noalloc: decode attention that allocates nothing, for
    callers that cannot call cudaMalloc when they run it (global-mode graph
    capture, fixed-pool runtimes, allocator hooks).  Device buffers only;
    queued on `stream` without waiting."""
    _check(lib().tg_attention_noalloc(C.c_void_p(stream), _ptr(q), _ptr(k_cache),
                                      _ptr(v_cache), dtype, n_seqs, max_ctx, n_head,
                                      n_kv_head, head_dim, _ptr(past_len), _ptr(out),
                                      _ptr(device_status)))


def comm_unique_id() -> bytes:
    buf = (C.c_char * 128)()
    _check(lib().tg_comm_unique_id(buf, 128))
    return bytes(buf)


class CudaBackend:
    """One device context: the counterpart of metal_backend::Context."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        _check(lib().tg_init(device, C.byref(h)))
        self._h = h
        self.device = device

    # -- lifetime (metal_backend::init / shutdown) -------------------------
    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def shutdown(self) -> None:
        if self._h:
            _check(lib().tg_shutdown(self._h))
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.shutdown()

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                lib().tg_shutdown(self._h)
        except Exception:
            pass

    # -- stream / batches (metal_batch_begin / metal_batch_end) -------------
    def set_stream(self, cuda_stream: int) -> None:
        _check(lib().tg_set_stream(self._h, C.c_void_p(cuda_stream)))

    def stream(self) -> int:
        s = C.c_void_p()
        _check(lib().tg_get_stream(self._h, C.byref(s)))
        return s.value or 0

    def num_sms(self) -> int:
        n = C.c_int()
        _check(lib().tg_device_sms(self._h, C.byref(n)))
        return n.value

    def metal_batch_begin(self) -> None:
        _check(lib().tg_batch_begin(self._h))

    def metal_batch_end(self) -> None:
        _check(lib().tg_batch_end(self._h))

    batch_begin = metal_batch_begin
    batch_end = metal_batch_end

    def synchronize(self) -> None:
        _check(lib().tg_synchronize(self._h))

    # -- CUDA graphs ----------------------------------------------------------
    def graph_begin(self) -> None:
        _check(lib().tg_graph_begin(self._h))

    def graph_end(self) -> "Graph":
        g = C.c_void_p()
        _check(lib().tg_graph_end(self._h, C.byref(g)))
        return Graph(self, g)

    def launch_count(self) -> int:
        n = C.c_longlong()
        _check(lib().tg_launch_count(self._h, C.byref(n)))
        return n.value

    def profile_enable(self, on=True) -> None:
        """True / PROFILE_ATTENTION: attention kernels; PROFILE_PROJECTION:
        the Q/K/V projection kernel; False: off."""
        mask = on if isinstance(on, int) and not isinstance(on, bool) else (1 if on else 0)
        _check(lib().tg_profile_enable(self._h, mask))

    def profile_read(self):
        """(summed decode-kernel milliseconds, timed launches)."""
        ms, n = C.c_double(), C.c_longlong()
        _check(lib().tg_profile_read(self._h, C.byref(ms), C.byref(n)))
        return ms.value, n.value

    def profile_read_stamps(self) -> np.ndarray:
        """%globaltimer stamps of the recorded bf16 decode steps
        (PROFILE_STAMPS): uint64 [step][row][4] in ns; decode CTA c in row
        c, merge CTA m in row num_sms() + m, absent CTAs 0."""
        n, rows = C.c_int(), C.c_int()
        cap = 1024 * 3 * self.num_sms() * 4
        buf = np.zeros(cap, np.uint64)
        _check(lib().tg_profile_read_stamps(self._h, buf.ctypes.data, cap, C.byref(n),
                                            C.byref(rows)))
        return buf[: n.value * rows.value * 4].reshape(n.value, rows.value, 4)

    # -- host-array mirrors (wrap_buffer) -----------------------------------
    def register_host(self, arr, flags: int = REGION_MIRROR) -> None:
        _check(lib().tg_register_host(self._h, _ptr(arr), arr.nbytes, flags))

    def unregister_host(self, arr) -> None:
        _check(lib().tg_unregister_host(self._h, _ptr(arr)))

    def region_sync(self, arr, to_device: bool = False) -> None:
        _check(lib().tg_region_sync(self._h, _ptr(arr), arr.nbytes,
                                    1 if to_device else 0))

    # -- reference-compatible ops ------------------------------------------
    def rope_op(self, data, n_heads: int, head_dim: int, pos: int,
                base: float = ROPE_BASE) -> None:
        """metal_backend::rope_op (metal_backend.hpp:381)."""
        _check(lib().tg_rope_op(self._h, _ptr(data), n_heads, head_dim, pos,
                                base))

    def elem_op(self, op: int, data, aux, dim: int) -> None:
        """metal_backend::elem_op (metal_backend.hpp:354), ops 0 and 2."""
        _check(lib().tg_elem_op(self._h, op, _ptr(data), _ptr(aux), dim))

    def attention_op(self, Q, K_cache, V_cache, output, n_head: int,
                     n_kv_head: int, head_dim: int, past_len: int) -> None:
        """metal_backend::attention_op (metal_backend.hpp:413)."""
        _check(lib().tg_attention_op(self._h, _ptr(Q), _ptr(K_cache),
                                     _ptr(V_cache), _ptr(output), n_head,
                                     n_kv_head, head_dim, past_len))

    def fused_qkv_op(self, W_q, W_k, W_v, x, y_q, y_k, y_v, q_rows: int,
                     k_rows: int, v_rows: int, cols: int, v_is_q8: bool) -> None:
        """metal_backend::fused_qkv_op (metal_backend.hpp:456): y_m = W_m x,
        W_q / W_k Q5_0, W_v Q5_0 or Q8_0."""
        _check(lib().tg_fused_qkv_op(self._h, _ptr(W_q), _ptr(W_k), _ptr(W_v),
                                     _ptr(x), _ptr(y_q), _ptr(y_k), _ptr(y_v),
                                     q_rows, k_rows, v_rows, cols,
                                     1 if v_is_q8 else 0))

    def attn_output(self, wtype: int, w_o, rows: int, cols: int, context, hidden,
                    n_seqs: int = 1) -> None:
        """hidden += W_o context (tg_attn_output; tmac_gguf.cpp:1497-1499)."""
        _check(lib().tg_attn_output(self._h, n_seqs, wtype, _ptr(w_o), rows, cols,
                                    _ptr(context), _ptr(hidden)))

    def matmul_q(self, wtype: int, rows: int, cols: int, w, x, y) -> None:
        """metal_backend::matmul_q5_0 / matmul_q8_0 (metal_backend.hpp:320-338)."""
        _check(lib().tg_matmul_q(self._h, wtype, rows, cols, _ptr(w), _ptr(x), _ptr(y)))

    # -- split-KV communicator ----------------------------------------------
    def comm_init(self, uid: bytes, rank: int, world: int,
                  timeout_ms: int = 60000) -> None:
        buf = C.create_string_buffer(uid, 128)
        _check(lib().tg_comm_init(self._h, buf, rank, world, timeout_ms))

    def set_wait_limit_ms(self, ms: int) -> None:
        """Bound of the split-KV kernels' in-kernel waits
        (tg_comm_set_wait_limit_ms); on expiry the next synchronisation
        raises TGError with TG_ERR_DEVICE."""
        _check(lib().tg_comm_set_wait_limit_ms(self._h, int(ms)))

    def set_exchange(self, exchange: int) -> None:
        """EXCHANGE_AUTO / EXCHANGE_PEER / EXCHANGE_NCCL (collective: the same
        value on every rank before the next split-KV call)."""
        _check(lib().tg_comm_set_exchange(self._h, exchange))

    @property
    def exchange(self) -> int:
        """The exchange the last split-KV call used."""
        v = C.c_int()
        _check(lib().tg_comm_exchange(self._h, C.byref(v)))
        return v.value

    def comm_destroy(self) -> None:
        _check(lib().tg_comm_destroy(self._h))

    def merge_records(self, records, out, n_parts: int, n_seqs: int,
                      n_head: int = N_HEAD, head_dim: int = HEAD_DIM) -> None:
        """Combine [n_parts][n_seqs][n_head*(head_dim+2)] softmax records."""
        _check(lib().tg_merge_records(self._h, n_parts, n_seqs, n_head,
                                      head_dim, _ptr(records), _ptr(out)))


class Graph:
    """A captured sequence of device-pointer calls (tg_graph_*)."""

    def __init__(self, backend: CudaBackend, handle: C.c_void_p):
        self.backend = backend
        self._h = handle

    def launch(self) -> None:
        _check(lib().tg_graph_launch(self.backend.handle, self._h))

    def destroy(self) -> None:
        if self._h and self.backend.handle:
            _check(lib().tg_graph_destroy(self._h))
        self._h = C.c_void_p()

    def __del__(self):
        try:
            if getattr(self, "_h", None) and self.backend.handle:
                lib().tg_graph_destroy(self._h)
        except Exception:
            pass


class KVCache:
    """Device-resident K/V caches [n_layers][n_seqs][max_ctx][n_kv*head_dim]
    (the static g_k_cache / g_v_cache of tmac_gguf.cpp:200-201, per
    sequence, optionally bf16, optionally one shard of a split context)."""

    def __init__(self, backend: CudaBackend, n_layers: int, n_seqs: int,
                 max_ctx: int, n_head: int = N_HEAD, n_kv_head: int = N_KV_HEAD,
                 head_dim: int = HEAD_DIM, dtype: int = DTYPE_F32,
                 shard_start: int = 0, global_ctx: int = 0,
                 rope_base: float = ROPE_BASE):
        self.backend = backend
        self.desc = tg_kv_desc(n_layers, n_seqs, max_ctx, n_head, n_kv_head,
                               head_dim, dtype, shard_start, global_ctx,
                               rope_base)
        h = C.c_void_p()
        _check(lib().tg_kv_create(backend.handle, C.byref(self.desc),
                                  C.byref(h)))
        self._h = h
        self.n_layers, self.n_seqs, self.max_ctx = n_layers, n_seqs, max_ctx
        self.n_head, self.n_kv_head, self.head_dim = n_head, n_kv_head, head_dim
        self.dtype = dtype
        self.shard_start = shard_start
        self.row = n_kv_head * head_dim

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def destroy(self) -> None:
        # After the backend's shutdown the C side has freed the cache already.
        if self._h and self.backend.handle:
            _check(lib().tg_kv_destroy(self._h))
        self._h = C.c_void_p()

    def __del__(self):
        try:
            if getattr(self, "_h", None) and self.backend.handle:
                lib().tg_kv_destroy(self._h)
        except Exception:
            pass

    def reset(self) -> None:
        _check(lib().tg_kv_reset(self._h))

    def layer_ptrs(self, layer: int):
        k, v = C.c_void_p(), C.c_void_p()
        _check(lib().tg_kv_layer_ptrs(self._h, layer, C.byref(k), C.byref(v)))
        return k.value, v.value

    def uses_tensor_cores(self) -> bool:
        n = C.c_int()
        _check(lib().tg_kv_uses_tensor_cores(self._h, C.byref(n)))
        return bool(n.value)

    def fill_normal(self, seed: int) -> None:
        _check(lib().tg_kv_fill_normal(self._h, seed & 0xFFFFFFFFFFFFFFFF))

    def write_rows(self, layer: int, seq: int, row0: int, k_rows, v_rows) -> None:
        k = np.ascontiguousarray(k_rows, dtype=np.float32) if isinstance(k_rows, np.ndarray) else k_rows
        v = np.ascontiguousarray(v_rows, dtype=np.float32) if isinstance(v_rows, np.ndarray) else v_rows
        n = (k.size if isinstance(k, np.ndarray) else v.size) // self.row
        _check(lib().tg_kv_write_rows(self._h, layer, seq, row0, n, _ptr(k),
                                      _ptr(v)))

    def read_rows(self, layer: int, seq: int, row0: int, n_rows: int):
        """Raw rows as float32 (fp32 cache) or uint16 bf16 bit patterns."""
        dt = np.float32 if self.dtype == DTYPE_F32 else np.uint16
        k = np.empty((n_rows, self.row), dtype=dt)
        v = np.empty((n_rows, self.row), dtype=dt)
        _check(lib().tg_kv_read_rows(self._h, layer, seq, row0, n_rows,
                                     _ptr(k), _ptr(v)))
        return k, v

    # -- decode ---------------------------------------------------------------
    def rope_cache_write(self, layer: int, q, k_new, v_new, pos) -> None:
        n = len(pos)
        pos = _as_i32(pos)
        _check(lib().tg_rope_cache_write(self.backend.handle, self._h, layer,
                                         n, _ptr(q), _ptr(k_new), _ptr(v_new),
                                         _ptr(pos)))

    def attention(self, layer: int, q, past_len, out) -> None:
        n = len(past_len)
        past_len = _as_i32(past_len)
        _check(lib().tg_attention_batched(self.backend.handle, self._h, layer,
                                          n, _ptr(q), _ptr(past_len), _ptr(out)))

    def decode_layer(self, layer: int, q, k_new, v_new, pos, out) -> None:
        n = len(pos)
        pos = _as_i32(pos)
        _check(lib().tg_decode_layer(self.backend.handle, self._h, layer, n,
                                     _ptr(q), _ptr(k_new), _ptr(v_new),
                                     _ptr(pos), _ptr(out)))

    def qkv_rope_cache_write(self, layer: int, weights: "QKVWeights", x, pos,
                             q_out) -> None:
        """Projection + bias + RoPE + cache-write from x (tg_qkv_rope_cache_write)."""
        n = len(pos)
        pos = _as_i32(pos)
        _check(lib().tg_qkv_rope_cache_write(self.backend.handle, self._h, layer, n,
                                             C.byref(weights.desc), _ptr(x), _ptr(pos),
                                             _ptr(q_out)))

    def decode_layer_x(self, layer: int, weights: "QKVWeights", x, pos, out) -> None:
        """The layer from the normed hidden state x to the attention output
        (tg_decode_layer_x)."""
        n = len(pos)
        pos = _as_i32(pos)
        _check(lib().tg_decode_layer_x(self.backend.handle, self._h, layer, n,
                                       C.byref(weights.desc), _ptr(x), _ptr(pos), _ptr(out)))

    def attention_block(self, layer: int, weights: "QKVWeights", w_o, x, pos, hidden,
                        o_type: int = WTYPE_Q5_0, split: bool = False) -> None:
        """x -> projection -> attention -> hidden += W_o context
        (tg_attention_block / tg_attention_block_splitkv)."""
        n = len(pos)
        pos = _as_i32(pos)
        fn = lib().tg_attention_block_splitkv if split else lib().tg_attention_block
        _check(fn(self.backend.handle, self._h, layer, n, C.byref(weights.desc), o_type,
                  _ptr(w_o), _ptr(x), _ptr(pos), _ptr(hidden)))

    def decode_layer_splitkv_x(self, layer: int, weights: "QKVWeights", x, pos,
                               out) -> None:
        """The layer from x on a split-KV shard (tg_decode_layer_splitkv_x)."""
        n = len(pos)
        pos = _as_i32(pos)
        _check(lib().tg_decode_layer_splitkv_x(self.backend.handle, self._h, layer, n,
                                               C.byref(weights.desc), _ptr(x), _ptr(pos),
                                               _ptr(out)))

    def attention_splitkv(self, layer: int, q, past_len, out) -> None:
        n = len(past_len)
        past_len = _as_i32(past_len)
        _check(lib().tg_attention_splitkv(self.backend.handle, self._h, layer,
                                          n, _ptr(q), _ptr(past_len), _ptr(out)))

    def prefill(self, layer: int, n_seqs: int, S: int, q, k, v, out) -> None:
        """Causal prefill of positions 0..S-1 (tg_prefill_layer)."""
        _check(lib().tg_prefill_layer(self.backend.handle, self._h, layer, n_seqs,
                                      S, _ptr(q), _ptr(k), _ptr(v), _ptr(out)))

    def attention_records(self, layer: int, q, past_len, records) -> None:
        """Softmax records of this shard (see tg_attention_records)."""
        n = len(past_len)
        past_len = _as_i32(past_len)
        _check(lib().tg_attention_records(self.backend.handle, self._h, layer,
                                          n, _ptr(q), _ptr(past_len),
                                          _ptr(records)))

    def record_floats(self) -> int:
        return self.n_head * (self.head_dim + 2)

    def decode_layer_splitkv(self, layer: int, q, k_new, v_new, pos, out) -> None:
        n = len(pos)
        pos = _as_i32(pos)
        _check(lib().tg_decode_layer_splitkv(self.backend.handle, self._h,
                                             layer, n, _ptr(q), _ptr(k_new),
                                             _ptr(v_new), _ptr(pos), _ptr(out)))


def _as_i32(x):
    if isinstance(x, np.ndarray):
        return np.ascontiguousarray(x, dtype=np.int32)
    if hasattr(x, "data_ptr"):
        return x
    return np.ascontiguousarray(np.asarray(x), dtype=np.int32)


class QKVWeights:
    """One layer's projection weights for tg_qkv_rope_cache_write /
    tg_decode_layer_x: block arrays (numpy uint8 or device tensors / device
    addresses) and optional fp32 biases.  The arrays are kept referenced."""

    def __init__(self, w_q, w_k, w_v, cols: int, q_type: int = WTYPE_Q5_0,
                 k_type: int = WTYPE_Q5_0, v_type: int = WTYPE_Q5_0,
                 b_q=None, b_k=None, b_v=None):
        self._keep = (w_q, w_k, w_v, b_q, b_k, b_v)
        self.desc = tg_qkv_weights(q_type, k_type, v_type, cols, _ptr(w_q), _ptr(w_k),
                                   _ptr(w_v), _ptr(b_q), _ptr(b_k), _ptr(b_v))


class Model:
    """A TMAC model file in device memory (tg_model_load_tmac: load_tmac,
    tmac_gguf.cpp:1372-1425)."""

    def __init__(self, backend: CudaBackend, path: str):
        self.backend = backend
        h = C.c_void_p()
        _check(lib().tg_model_load_tmac(backend.handle, os.fsencode(path), C.byref(h)))
        self._h = h

    def __len__(self) -> int:
        n = C.c_int()
        _check(lib().tg_model_count(self._h, C.byref(n)))
        return n.value

    @staticmethod
    def _info(t: tg_tensor_info):
        if not t.name:
            return None
        return {"name": t.name.decode(errors="replace"), "rows": t.rows, "cols": t.cols,
                "n_bytes": t.n_bytes, "type": t.type, "data": t.data}

    def tensor(self, index: int):
        t = tg_tensor_info()
        _check(lib().tg_model_tensor_at(self._h, index, C.byref(t)))
        return self._info(t)

    def find(self, name: str):
        """get_tensor_info (tmac_gguf.cpp:417-422); None when absent."""
        t = tg_tensor_info()
        _check(lib().tg_model_find(self._h, name.encode(), C.byref(t)))
        return self._info(t)

    def read(self, index: int) -> bytes:
        info = self.tensor(index)
        buf = C.create_string_buffer(max(int(info["n_bytes"]), 1))
        _check(lib().tg_model_read(self._h, index, buf, int(info["n_bytes"])))
        return buf.raw[:int(info["n_bytes"])]

    def layer_attention(self, layer: int):
        """(QKVWeights, w_o device address or None, o_type) of one layer."""
        d = tg_qkv_weights()
        wo = C.c_void_p()
        ot = C.c_int()
        _check(lib().tg_model_layer_attention(self._h, layer, C.byref(d), C.byref(wo),
                                              C.byref(ot)))
        w = QKVWeights.__new__(QKVWeights)
        w._keep = (self,)
        w.desc = d
        return w, wo.value, ot.value

    def destroy(self) -> None:
        if self._h:
            _check(lib().tg_model_destroy(self._h))
        self._h = C.c_void_p()

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                lib().tg_model_destroy(self._h)
        except Exception:
            pass
