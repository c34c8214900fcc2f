"""ctypes binding of ``include/shk_cuda.h`` (libshk_cuda.so).

Device buffers are passed as integer addresses (e.g. ``torch.Tensor.data_ptr()``).
The library must be built in-tree (``python -m shukuchi_b200.build``); there is
no fallback when it is missing or when a call fails.
"""
from __future__ import annotations

import ctypes as C
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libshk_cuda.so")
HEADER = os.path.join(os.path.dirname(_HERE), "include", "shk_cuda.h")

SHK_OK = 0
FLAG_PERSISTENT = 2  # SHK_CUDA_FLAG_PERSISTENT: whole-token steps in the persistent decode kernel
FLAG_NO_PDL = 4  # SHK_CUDA_FLAG_NO_PDL: decode-step graphs without programmatic dependent launch
STATUS = {0: "SHK_OK", -1: "SHK_EINVAL", -2: "SHK_ENOMEM", -3: "SHK_ECUDA", -4: "SHK_EUNSUPPORTED",
          -5: "SHK_ETIMEOUT", -6: "SHK_ENODEV", -7: "SHK_ENCCL", -8: "SHK_EDEVICE"}


class ShkError(RuntimeError):
    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} failed: {STATUS.get(code, code)}")
        self.code = code


class CudaConfig(C.Structure):
    _fields_ = [("device", C.c_int), ("flags", C.c_uint32)]


class KvConfig(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("block_size", C.c_uint32), ("max_seq_len", C.c_uint32)]


class ModelDesc(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("n_embd", C.c_uint32), ("n_heads", C.c_uint32),
                ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("n_ff", C.c_uint32),
                ("n_vocab", C.c_uint32), ("rope_theta", C.c_float),
                ("tok_embd_dev", C.c_void_p), ("tok_embd_dtype", C.c_uint32),
                ("output_dev", C.c_void_p), ("output_dtype", C.c_uint32)]


class LayerDesc(C.Structure):
    _fields_ = [("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p),
                ("attn_q", C.c_void_p), ("attn_k", C.c_void_p), ("attn_v", C.c_void_p),
                ("attn_o", C.c_void_p), ("ffn_gate", C.c_void_p), ("ffn_up", C.c_void_p),
                ("ffn_down", C.c_void_p),
                ("attn_q_dtype", C.c_uint32), ("attn_k_dtype", C.c_uint32),
                ("attn_v_dtype", C.c_uint32), ("attn_o_dtype", C.c_uint32),
                ("ffn_gate_dtype", C.c_uint32), ("ffn_up_dtype", C.c_uint32),
                ("ffn_down_dtype", C.c_uint32),
                ("row_stride_v", C.c_uint32), ("row_stride_down", C.c_uint32)]


P, U32, U64, I, F, SZ = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int, C.c_float, C.c_size_t
_SIGS = {
    "shk_cuda_init": (P, [C.POINTER(CudaConfig)]),
    "shk_cuda_shutdown": (None, [P]),
    "shk_cuda_available": (I, []),
    "shk_cuda_report": (None, [P]),
    "shk_cuda_check": (I, [P]),
    "shk_cuda_strerror": (C.c_char_p, [I]),
    "shk_cuda_stream": (P, [P]),
    "shk_cuda_num_sms": (I, [P]),
    "shk_cuda_dev_alloc": (I, [P, SZ, C.POINTER(P)]),
    "shk_cuda_dev_free": (I, [P, P]),
    "shk_cuda_host_alloc": (I, [P, SZ, C.POINTER(P)]),
    "shk_cuda_host_free": (I, [P, P]),
    "shk_cuda_memcpy_h2d": (I, [P, P, P, SZ, P]),
    "shk_cuda_memcpy_d2h": (I, [P, P, P, SZ, P]),
    "shk_cuda_sync": (I, [P, P]),
    "shk_cuda_matmul_q4k_vec": (I, [P, P, P, P, U32, U32, P]),
    "shk_cuda_matmul_q6k_vec": (I, [P, P, P, P, U32, U32, P]),
    "shk_cuda_matmul_q5k_vec": (I, [P, P, P, P, U32, U32, P]),
    "shk_cuda_prefill": (I, [P, P, U32, U32, P, P, P]),
    "shk_cuda_matmul_q4k_vec_host": (I, [P, P, P, P, U32, U32]),
    "shk_cuda_matmul_q6k_vec_host": (I, [P, P, P, P, U32, U32]),
    "shk_cuda_matmul_q5k_vec_host": (I, [P, P, P, P, U32, U32]),
    "shk_cuda_rmsnorm": (I, [P, P, P, P, U32, P]),
    "shk_cuda_rope": (I, [P, P, U32, U32, U32, F, P]),
    "shk_cuda_swiglu": (I, [P, P, P, P, U32, P]),
    "shk_cuda_embed": (I, [P, P, U32, U32, U32, P, U32, P]),
    "shk_cuda_argmax": (I, [P, P, U32, C.POINTER(U32)]),
    "shk_cuda_argmax_noalloc": (I, [P, U32, P, P]),
    "shk_cuda_selftest_wait_timeout": (I, [P, U32]),
    "shk_cuda_q6k_repack": (I, [P, P, U32, U32, U32, I, P]),
    "shk_cuda_layer_stage_q6k_planar": (I, [P, U32, P, U32, U32, U32]),
    "shk_cuda_matvec": (I, [P, U32, P, U32, P, P, U32, U32, P]),
    "shk_cuda_tiled_bytes": (SZ, [U32, U32, U32]),
    "shk_cuda_tile": (I, [P, U32, P, U32, U32, U32, P, P]),
    "shk_cuda_prefill_matmul": (I, [P, U32, P, U32, P, P, U32, U32, U32, P]),
    "shk_cuda_tp_unique_id": (I, [P, SZ]),
    "shk_cuda_tp_init": (I, [P, I, I, P]),
    "shk_cuda_tp_comm_size": (I, [P]),
    "shk_cuda_model_set_tp_rows": (I, [P, U32, U32, U32, U32]),
    "shk_cuda_model_tp_p2p_export": (I, [P, P, SZ]),
    "shk_cuda_model_tp_p2p_import": (I, [P, P, P]),
    "shk_cuda_model_tp_ll_export": (I, [P, P, SZ]),
    "shk_cuda_model_tp_ll_import": (I, [P, P]),
    "shk_cuda_kv_create": (P, [P, C.POINTER(KvConfig)]),
    "shk_cuda_kv_destroy": (None, [P]),
    "shk_cuda_kv_append": (I, [P, U32, U32, P, P, P]),
    "shk_cuda_kv_append_range": (I, [P, U32, U32, U32, P, P, P]),
    "shk_cuda_kv_read_range": (I, [P, U32, U32, U32, P, P, P]),
    "shk_cuda_kv_read_blocks": (I, [P, U32, U32, U32, P, P, P]),
    "shk_cuda_kv_attend": (I, [P, U32, P, P, P, P, U32, U32, F, P]),
    "shk_cuda_kv_attend_batch": (I, [P, U32, U32, P, P, P, P, U32, U32, F, P]),
    "shk_cuda_kv_clear": (None, [P]),
    "shk_cuda_kv_seq_len": (U32, [P, U32]),
    "shk_cuda_model_create": (P, [P, C.POINTER(ModelDesc), P]),
    "shk_cuda_model_destroy": (None, [P]),
    "shk_cuda_model_set_layer": (I, [P, U32, C.POINTER(LayerDesc)]),
    "shk_cuda_forward_layer": (I, [P, C.POINTER(LayerDesc), U32, U32, P, P]),
    "shk_cuda_model_embed": (I, [P, U32, P]),
    "shk_cuda_model_lm_head": (I, [P, C.POINTER(U32), P, P]),
    "shk_cuda_model_hidden": (P, [P]),
    "shk_cuda_token_step": (I, [P, U32, U32, I, C.POINTER(U32), P]),
    "shk_cuda_decode_steps": (I, [P, U32, U32, U32, P]),
    "shk_cuda_model_token": (I, [P, C.POINTER(U32)]),
    "shk_cuda_model_trace_enable": (I, [P, U32]),
    "shk_cuda_model_trace_read": (I, [P, C.POINTER(U64), U32]),
    "shk_cuda_model_launch_part": (I, [P, U32, U32, P, C.POINTER(U64)]),
    "shk_cuda_layer_stage": (I, [P, U32, P, P, SZ]),
    "shk_cuda_layer_stage_rows": (I, [P, U32, P, SZ, P, SZ, SZ]),
    "shk_cuda_layer_stage_2d": (I, [P, U32, P, C.c_size_t, P, C.c_size_t, C.c_size_t, C.c_size_t]),
    "shk_cuda_layer_commit": (I, [P, U32]),
    "shk_cuda_layer_ready": (I, [P, U32, I]),
    "shk_cuda_layer_wait": (I, [P, U32, P]),
    "shk_cuda_layer_release": (I, [P, U32, P]),
}

_lib = None


def header_functions(path: str = HEADER) -> list[str]:
    """Names of the functions include/shk_cuda.h declares."""
    txt = open(path).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(shk_cuda_\w+)\s*\(", txt)))


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m shukuchi_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(fn: str, rc: int) -> int:
    if rc < 0:
        raise ShkError(fn, rc)
    return rc


def _call(name: str, *args) -> int:
    return check(name, getattr(lib(), name)(*args))


class Context:
    """A device context (shk_ctx): compute + copy streams, error word."""

    def __init__(self, device: int = 0, flags: int = 0):
        cfg = CudaConfig(device, flags)
        self.h = lib().shk_cuda_init(C.byref(cfg))
        if not self.h:
            raise ShkError("shk_cuda_init", -6)

    def close(self) -> None:
        if self.h:
            lib().shk_cuda_shutdown(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def stream(self) -> int:
        return lib().shk_cuda_stream(self.h)

    @property
    def num_sms(self) -> int:
        return lib().shk_cuda_num_sms(self.h)

    def check(self) -> None:
        _call("shk_cuda_check", self.h)

    def sync(self, stream: int | None = None) -> None:
        _call("shk_cuda_sync", self.h, stream)

    def report(self) -> None:
        lib().shk_cuda_report(self.h)

    def q6k_repack(self, w_dev: int, rows: int, k: int, row_stride: int = 0, to_planar: bool = True,
                   stream: int | None = None) -> None:
        """Q6_K rows in place between the GGUF and the planar layout."""
        _call("shk_cuda_q6k_repack", self.h, w_dev, rows, k, row_stride, 1 if to_planar else 0, stream)

    def tile(self, dtype: int, src_dev: int, rows: int, k: int, dst_dev: int, src_row_stride: int = 0,
             stream: int | None = None) -> None:
        """GGUF rows (dtype 12 / 14) -> the row-tiled layout at dst_dev
        (tiled_bytes(dtype, rows, k) bytes)."""
        _call("shk_cuda_tile", self.h, dtype, src_dev, src_row_stride, rows, k, dst_dev, stream)

    def matvec(self, dtype: int, w_dev: int, x_dev: int, y_dev: int, m: int, k: int, row_stride: int = 0,
               stream: int | None = None) -> None:
        _call("shk_cuda_matvec", self.h, dtype, w_dev, row_stride, x_dev, y_dev, m, k, stream)

    def prefill_matmul(self, dtype: int, w_dev: int, x_dev: int, y_dev: int, m: int, k: int, n_tokens: int,
                       row_stride: int = 0, stream: int | None = None) -> None:
        """y[t][r] = sum_k W[r][k] x[t][k] on the tensor cores (f16 inputs, each token row
        scaled by a power of two)."""
        _call("shk_cuda_prefill_matmul", self.h, dtype, w_dev, row_stride, x_dev, y_dev, m, k, n_tokens, stream)

    def tp_init(self, rank: int, world: int, uid: bytes) -> None:
        """Joins this context to a tensor-parallel group of `world` ranks
        (one process or thread per GPU); uid comes from tp_unique_id() on rank 0."""
        buf = C.create_string_buffer(bytes(uid), len(uid))
        _call("shk_cuda_tp_init", self.h, rank, world, buf)

    def tp_comm_size(self) -> int:
        """Ranks in this context's NCCL communicator (1 without one)."""
        return _call("shk_cuda_tp_comm_size", self.h)

    def matmul(self, qtype: int, w_dev: int, x_dev: int, y_dev: int, m: int, k: int,
               stream: int | None = None) -> None:
        name = {12: "shk_cuda_matmul_q4k_vec", 13: "shk_cuda_matmul_q5k_vec", 14: "shk_cuda_matmul_q6k_vec"}[qtype]
        _call(name, self.h, w_dev, x_dev, y_dev, m, k, stream)

    def matmul_host(self, qtype: int, w, x, y, m: int, k: int) -> None:
        """Host-pointer, synchronous variant (numpy arrays)."""
        name = {12: "shk_cuda_matmul_q4k_vec_host", 13: "shk_cuda_matmul_q5k_vec_host",
                14: "shk_cuda_matmul_q6k_vec_host"}[qtype]
        _call(name, self.h, w.ctypes.data, x.ctypes.data, y.ctypes.data, m, k)

    def rmsnorm(self, x, w, y, d, stream=None):
        _call("shk_cuda_rmsnorm", self.h, x, w, y, d, stream)

    def rope(self, qk, n_heads, head_dim, pos, theta, stream=None):
        _call("shk_cuda_rope", self.h, qk, n_heads, head_dim, pos, theta, stream)

    def swiglu(self, g, u, h, n, stream=None):
        _call("shk_cuda_swiglu", self.h, g, u, h, n, stream)

    def embed(self, table, dtype, n_vocab, token, out, n_embd, stream=None):
        _call("shk_cuda_embed", self.h, table, dtype, n_vocab, token, out, n_embd, stream)

    def argmax(self, x, n) -> int:
        out = C.c_uint32(0)
        _call("shk_cuda_argmax", self.h, x, n, C.byref(out))
        return out.value

    # staging
    def layer_stage(self, slot, dst_dev, src_host_ptr, nbytes):
        _call("shk_cuda_layer_stage", self.h, slot, dst_dev, src_host_ptr, nbytes)

    def layer_stage_rows(self, slot, dst_dev, dst_row, src_host_ptr, src_row, rows):
        _call("shk_cuda_layer_stage_rows", self.h, slot, dst_dev, dst_row, src_host_ptr, src_row, rows)

    def layer_commit(self, slot):
        _call("shk_cuda_layer_commit", self.h, slot)

    def layer_ready(self, slot, wait=False) -> bool:
        return bool(_call("shk_cuda_layer_ready", self.h, slot, 1 if wait else 0))

    def layer_wait(self, slot, stream=None):
        _call("shk_cuda_layer_wait", self.h, slot, stream)


DTYPE_Q6_K_PLANAR = 0x10E
DTYPE_Q4_K_TILED = 0x20C
DTYPE_Q6_K_TILED = 0x20E


def tiled_bytes(dtype: int, rows: int, k: int) -> int:
    """Bytes of the row-tiled form of a rows x k matrix (0 if not tileable)."""
    return int(lib().shk_cuda_tiled_bytes(dtype, rows, k))


def tp_unique_id() -> bytes:
    """A new communicator id for shk_cuda_tp_init (created on rank 0)."""
    buf = C.create_string_buffer(128)
    n = check("shk_cuda_tp_unique_id", lib().shk_cuda_tp_unique_id(buf, 128))
    return buf.raw[:n]


class KvCache:
    """Q8_0 KV cache in HBM (shk_kv)."""

    def __init__(self, ctx: Context, n_layers, n_kv_heads, head_dim, max_seq_len, block_size=32):
        self.ctx = ctx
        cfg = KvConfig(n_layers, n_kv_heads, head_dim, block_size, max_seq_len)
        self.h = lib().shk_cuda_kv_create(ctx.h, C.byref(cfg))
        if not self.h:
            raise ShkError("shk_cuda_kv_create", -2)
        self.n_layers, self.n_kv, self.hd, self.max_seq = n_layers, n_kv_heads, head_dim, max_seq_len

    def close(self):
        if self.h:
            lib().shk_cuda_kv_destroy(self.h)
            self.h = None

    def append(self, layer, pos, k, v, stream=None):
        _call("shk_cuda_kv_append", self.h, layer, pos, k, v, stream)

    def append_range(self, layer, start, n, k, v, stream=None):
        _call("shk_cuda_kv_append_range", self.h, layer, start, n, k, v, stream)

    def read_range(self, layer, start, end, k, v, stream=None):
        _call("shk_cuda_kv_read_range", self.h, layer, start, end, k, v, stream)

    def read_blocks(self, layer, start, end, k, v, stream=None):
        _call("shk_cuda_kv_read_blocks", self.h, layer, start, end, k, v, stream)

    def attend(self, layer, q, out, n_heads, seq_len, scale, k_new=None, v_new=None, stream=None):
        _call("shk_cuda_kv_attend", self.h, layer, q, k_new, v_new, out, n_heads, seq_len, scale, stream)

    def attend_batch(self, layer0, n_seq, q, out, n_heads, seq_len, scale, k_new=None, v_new=None,
                     stream=None):
        """attend for n_seq sequences (cache layers layer0..) in one launch."""
        _call("shk_cuda_kv_attend_batch", self.h, layer0, n_seq, q, k_new, v_new, out, n_heads, seq_len, scale,
              stream)

    def clear(self):
        lib().shk_cuda_kv_clear(self.h)

    def seq_len(self, layer) -> int:
        return lib().shk_cuda_kv_seq_len(self.h, layer)


class DeviceModel:
    """shk_model over device-resident weights."""

    def __init__(self, ctx: Context, kv: KvCache, desc: ModelDesc):
        self.ctx, self.kv, self.desc = ctx, kv, desc
        self.h = lib().shk_cuda_model_create(ctx.h, C.byref(desc), kv.h)
        if not self.h:
            raise ShkError("shk_cuda_model_create", -1)

    def close(self):
        if self.h:
            lib().shk_cuda_model_destroy(self.h)
            self.h = None

    def set_layer(self, layer: int, lv: LayerDesc):
        _call("shk_cuda_model_set_layer", self.h, layer, C.byref(lv))

    def set_tp_rows(self, o_lo: int, o_hi: int, v_lo: int, v_hi: int):
        _call("shk_cuda_model_set_tp_rows", self.h, o_lo, o_hi, v_lo, v_hi)

    def tp_p2p_export(self) -> bytes:
        """IPC handle of this rank's exchange buffer (peer-memory all-reduce)."""
        buf = C.create_string_buffer(64)
        n = check("shk_cuda_model_tp_p2p_export", lib().shk_cuda_model_tp_p2p_export(self.h, buf, 64))
        return buf.raw[:n]

    def tp_p2p_import(self, handles: list, o_ranges: list):
        """handles: every rank's export in rank order; o_ranges: every rank's
        (o_lo, o_hi)."""
        hb = C.create_string_buffer(b"".join(handles), 64 * len(handles))
        rg = (C.c_uint32 * (2 * len(o_ranges)))(*[v for r in o_ranges for v in r])
        _call("shk_cuda_model_tp_p2p_import", self.h, hb, rg)

    def tp_ll_export(self) -> bytes:
        """IPC handle of this rank's exchange buffer (all-reduce with flags in
        the data words)."""
        buf = C.create_string_buffer(64)
        n = check("shk_cuda_model_tp_ll_export", lib().shk_cuda_model_tp_ll_export(self.h, buf, 64))
        return buf.raw[:n]

    def tp_ll_import(self, handles: list):
        """handles: every rank's export in rank order."""
        hb = C.create_string_buffer(b"".join(handles), 64 * len(handles))
        _call("shk_cuda_model_tp_ll_import", self.h, hb)

    def forward_layer(self, lv: LayerDesc, layer, pos, hidden_dev, stream=None):
        _call("shk_cuda_forward_layer", self.h, C.byref(lv), layer, pos, hidden_dev, stream)

    def embed(self, token, stream=None):
        _call("shk_cuda_model_embed", self.h, token, stream)

    def lm_head(self, logits_host_ptr=None) -> int:
        t = C.c_uint32(0)
        _call("shk_cuda_model_lm_head", self.h, C.byref(t), logits_host_ptr, None)
        return t.value

    @property
    def hidden(self) -> int:
        return lib().shk_cuda_model_hidden(self.h)

    def token_step(self, token, pos, want_next=True, logits_host_ptr=None) -> int:
        t = C.c_uint32(0)
        _call("shk_cuda_token_step", self.h, token, pos, 1 if want_next else 0, C.byref(t), logits_host_ptr)
        return t.value

    def prefill(self, tokens, pos0=0, logits_host_ptr=None, stream=None) -> int:
        """Batched prompt prefill of `tokens` (uint32 numpy array) at positions
        pos0..; returns the argmax of the last row's logits."""
        import numpy as np
        t = np.ascontiguousarray(tokens, np.uint32)
        nx = C.c_uint32(0)
        _call("shk_cuda_prefill", self.h, t.ctypes.data, t.size, pos0, C.byref(nx), logits_host_ptr, stream)
        return nx.value

    def decode_steps(self, first_token, first_pos, n, stream=None):
        _call("shk_cuda_decode_steps", self.h, first_token, first_pos, n, stream)

    def launch_part(self, layer: int, part: int, stream=None) -> int:
        b = C.c_uint64(0)
        _call("shk_cuda_model_launch_part", self.h, layer, part, stream, C.byref(b))
        return b.value

    def trace_enable(self, n_phases: int):
        _call("shk_cuda_model_trace_enable", self.h, n_phases)

    def trace_read(self, cap: int):
        buf = (U64 * cap)()
        n = lib().shk_cuda_model_trace_read(self.h, buf, cap)
        check("shk_cuda_model_trace_read", min(n, 0))
        return list(buf[:n])

    def last_token(self) -> int:
        t = C.c_uint32(0)
        _call("shk_cuda_model_token", self.h, C.byref(t))
        return t.value
