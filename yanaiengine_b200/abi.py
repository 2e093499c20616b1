"""ctypes binding of include/yk.h (libyk.so) and include/yk_host.h (libyk_host.so).

The CUDA module is the only implementation: if the in-tree libraries are
missing this raises instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libyk.so"
HOST_LIB_PATH = PKG / "libyk_host.so"

YK_OK, YK_ERR_ARG, YK_ERR_OOM, YK_ERR_CUDA, YK_ERR_NCCL, YK_ERR_TIMEOUT, YK_ERR_DEVICE_CHECK, YK_ERR_UNSUPPORTED = range(8)
DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2  # F16: checkpoint sources only
LOAD_ROPE_HALF = 1
ACT_SILU, ACT_GELU_TANH = 0, 1
BLOCK_SIZE = 16
(T_EMBED, T_WQ, T_WK, T_WV, T_WO, T_WGATE, T_WUP, T_WDOWN, T_NORM1, T_NORM2, T_FINAL_NORM,
 T_LM_HEAD) = range(12)
LAYOUT_OUT_IN, LAYOUT_IN_OUT = 0, 1


class ModelConfig(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int32), ("d_model", C.c_int32), ("n_layers", C.c_int32), ("n_heads", C.c_int32),
        ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn_dim", C.c_int32),
        ("rope_theta", C.c_float), ("rms_eps", C.c_float), ("attn_cap", C.c_float), ("final_cap", C.c_float),
        ("window", C.c_int32), ("window_layer_parity", C.c_int32), ("act", C.c_int32), ("ref_compat", C.c_int32),
        ("dtype", C.c_int32), ("max_tokens", C.c_int32), ("max_seqs", C.c_int32),
    ]

    def to_dict(self) -> dict:
        return {f: getattr(self, f) for f, _ in self._fields_}


def make_config(**kw) -> ModelConfig:
    defaults = dict(rope_theta=10000.0, rms_eps=1e-5, attn_cap=0.0, final_cap=0.0, window=0,
                    window_layer_parity=-1, act=ACT_SILU, ref_compat=0, dtype=DTYPE_BF16, max_tokens=256,
                    max_seqs=64)
    defaults.update(kw)
    c = ModelConfig()
    for k, v in defaults.items():
        setattr(c, k, v)
    return c


class YKError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"yk status {status}: {msg}")
        self.status = status


_P = C.c_void_p
_U32P = C.POINTER(C.c_uint32)
_I32P = C.POINTER(C.c_int32)
_F32P = C.POINTER(C.c_float)

_PROTOS = {
    "yk_last_error": (C.c_int32, [C.c_char_p, C.c_size_t]),
    "yk_engine_create": (C.c_int32, [C.c_int32, C.POINTER(_P)]),
    "yk_engine_destroy": (None, [_P]),
    "yk_engine_stream": (C.c_int32, [_P, C.POINTER(_P)]),
    "yk_engine_sync": (C.c_int32, [_P]),
    "yk_engine_device_error": (C.c_int32, [_P, _U32P]),
    "yk_engine_launch_count": (C.c_uint64, [_P]),
    "yk_engine_profile": (C.c_int32, [_P, C.c_int32]),
    "yk_engine_profile_read": (C.c_int32, [_P, C.c_int32, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                           C.POINTER(C.c_double), C.POINTER(C.c_int64)]),
    "yk_model_create": (C.c_int32, [_P, C.POINTER(ModelConfig), C.c_uint64, C.c_float, C.POINTER(_P)]),
    "yk_model_create_tp": (C.c_int32, [_P, C.POINTER(ModelConfig), C.c_int32, C.c_int32, C.c_uint64, C.c_float,
                                       C.POINTER(_P)]),
    "yk_tp_unique_id": (C.c_int32, [C.POINTER(C.c_uint8)]),
    "yk_tp_init": (C.c_int32, [_P, C.POINTER(C.c_uint8), C.c_int32, C.c_int32]),
    "yk_tp_init_timeout": (C.c_int32, [_P, C.POINTER(C.c_uint8), C.c_int32, C.c_int32, C.c_int64]),
    "yk_model_destroy": (None, [_P]),
    "yk_model_get_config": (C.c_int32, [_P, C.POINTER(ModelConfig)]),
    "yk_model_tensor_shape": (C.c_int32, [_P, C.c_int32, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "yk_model_set_tensor": (C.c_int32, [_P, C.c_int32, C.c_int32, _F32P, C.c_int32]),
    "yk_model_get_tensor": (C.c_int32, [_P, C.c_int32, C.c_int32, _F32P]),
    "yk_safetensors_open": (C.c_int32, [C.c_char_p, C.POINTER(_P)]),
    "yk_safetensors_close": (None, [_P]),
    "yk_safetensors_count": (C.c_int32, [_P]),
    "yk_safetensors_name": (C.c_int32, [_P, C.c_int32, C.POINTER(C.c_char_p)]),
    "yk_safetensors_info": (C.c_int32, [_P, C.c_char_p, C.c_void_p]),
    "yk_model_load_tensor": (C.c_int32, [_P, C.c_int32, C.c_int32, _P, C.c_int32, C.c_int64, C.c_int64,
                                         C.c_int32]),
    "yk_model_load_safetensors": (C.c_int32, [_P, C.POINTER(_P), C.c_int32, C.c_float, C.c_int32, _I32P]),
    "yk_hf_tensor_id": (C.c_int32, [C.c_char_p, C.c_int32, _I32P, _I32P]),
    "yk_kv_pool_create": (C.c_int32, [_P, C.POINTER(ModelConfig), C.c_int32, C.POINTER(_P)]),
    "yk_kv_pool_create_layers": (C.c_int32, [_P, C.POINTER(ModelConfig), C.c_int32, C.c_int32, C.POINTER(_P)]),
    "yk_forward_step_split": (C.c_int32, [_P, _P, _P, _U32P, C.c_int32, _U32P, _U32P, C.c_int32, _I32P, C.c_int32,
                                          _I32P, C.c_int32, C.c_int32, _P, C.c_int32, C.c_int32, _I32P]),
    "yk_kv_pool_destroy": (None, [_P]),
    "yk_kv_pool_num_blocks": (C.c_int32, [_P]),
    "yk_kv_pool_fill_random": (C.c_int32, [_P, C.c_uint64, C.c_float]),
    "yk_kv_pool_read_page": (C.c_int32, [_P, C.c_int32, C.c_int32, C.c_int32, _F32P]),
    "yk_forward_step": (C.c_int32, [_P, _P, _U32P, C.c_int32, _U32P, _U32P, C.c_int32, _I32P, C.c_int32,
                                    C.c_int32, _I32P]),
    "yk_forward_step_drafts": (C.c_int32, [_P, _P, _U32P, C.c_int32, _U32P, _U32P, C.c_int32, _I32P, C.c_int32,
                                    C.c_int32, _P, C.c_int32, C.c_int32, _I32P]),
    "yk_logits_copy_to_host": (C.c_int32, [_P, C.c_int32, C.c_int32, _F32P]),
    "yk_sampler_create": (C.c_int32, [_P, C.c_int32, C.c_int32, C.c_int32, C.POINTER(_P)]),
    "yk_sampler_destroy": (None, [_P]),
    "yk_draft_sample": (C.c_int32, [_P, _P, C.c_int32, C.c_int32, C.c_float, C.c_uint64, C.c_uint32, _U32P,
                                    _U32P]),
    "yk_spec_verify": (C.c_int32, [_P, _P, C.c_int32, C.c_float, C.c_uint64, C.c_uint32, _U32P, _U32P, _U32P,
                                   _I32P]),
    "yk_spec_verify_probs": (C.c_int32, [_P, C.c_int32, _F32P, _F32P, _U32P, C.c_uint64, C.c_uint32, _U32P,
                                         _U32P, _I32P]),
    "yk_spec_sample_logits": (C.c_int32, [_P, C.c_int32, _F32P, _F32P, C.c_float, C.c_uint64, C.c_uint32, _U32P,
                                          _U32P, _U32P, _I32P]),
    "yk_sampler_read_probs": (C.c_int32, [_P, C.c_int32, C.c_int32, _F32P]),
    "yk_sampler_read_drafts": (C.c_int32, [_P, C.c_int32, _U32P]),
    "yk_spec_verify_range": (C.c_int32, [_P, _P, C.c_int32, C.c_int32, C.c_float, C.c_uint64, C.c_uint32, _U32P, _U32P,
                                         _U32P, _I32P]),
    "yk_tp_allgather_u32": (C.c_int32, [_P, _U32P, C.c_int32, _U32P]),
    "yk_spec_verify_logits_noalloc": (C.c_int32, [C.c_int32, _P, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32,
                                                  C.c_float, C.c_uint64, C.c_uint32, _P, _P]),
    # include/yk_testing.h
    "ykt_gemm_bf16": (C.c_int32, [_P, C.POINTER(C.c_uint16), C.POINTER(C.c_uint16), C.c_int32, C.c_int32,
                                  C.c_int32, C.c_int32, _F32P]),
    "ykt_gemm_bf16_timed": (C.c_int32, [_P, C.POINTER(C.c_uint16), C.POINTER(C.c_uint16), C.c_int32, C.c_int32,
                                        C.c_int32, C.c_int32, C.c_int32, _F32P, _F32P, C.POINTER(C.c_uint64),
                                        _I32P]),
    "ykt_gemm_bf16_epi_timed": (C.c_int32, [_P, C.POINTER(C.c_uint16), C.POINTER(C.c_uint16), C.c_int32, C.c_int32,
                                            C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _F32P,
                                            C.POINTER(C.c_uint64), _I32P]),
    "ykt_attention_stamps_enable": (C.c_int32, [_P, C.c_int32]),
    "ykt_gemm_stamps_enable": (C.c_int32, [_P, C.c_uint32]),
    "ykt_gemm_stamps_read": (C.c_int32, [_P, C.POINTER(C.c_uint64), C.c_int32, _I32P]),
    "ykt_trace_enable": (C.c_int32, [_P, C.c_int32]),
    "ykt_sampler_stamps_enable": (C.c_int32, [_P, C.c_int32]),
    "ykt_sampler_stamps_read": (C.c_int32, [_P, C.POINTER(C.c_uint64), C.c_int32]),
    "ykt_wait_timeout": (C.c_int32, [_P, C.c_int32, C.POINTER(C.c_double)]),
    "ykt_tp_allreduce_timed": (C.c_int32, [_P, C.c_int64, C.c_int32, C.c_int32, C.POINTER(C.c_double),
                                           C.POINTER(C.c_uint64)]),
    "ykt_sampler_target_probs": (C.c_int32, [_P, C.c_int32, C.c_float, C.POINTER(C.c_float)]),
    "ykt_trace_read": (C.c_int32, [_P, C.POINTER(C.c_uint64), C.c_int32, C.POINTER(C.c_uint64)]),
    "ykt_attention_stamps_read": (C.c_int32, [_P, C.POINTER(C.c_uint64), C.c_int32, _I32P]),
}

_HOST_PROTOS = {
    "ykh_scheduler_create": (C.c_int32, [_P, _P, _P, _P, _P, C.c_int32, C.c_float, C.c_uint64, C.POINTER(_P)]),
    "ykh_scheduler_destroy": (None, [_P]),
    "ykh_scheduler_create_split": (C.c_int32, [_P, _P, _P, _P, _P, _P, _P, C.c_int32, C.c_float, C.c_uint64,
                                               C.POINTER(_P)]),
    "ykh_usage_windowed": (C.c_float, [_P, C.c_int32]),
    "ykh_submit": (C.c_int32, [_P, _U32P, C.c_int32, C.c_int32, C.c_int64, C.c_uint32]),
    "ykh_submit_cached": (C.c_int32, [_P, _U32P, C.c_int32, C.c_int32, C.c_int64, C.c_uint32]),
    "ykh_submit_stream": (C.c_int32, [_P, _U32P, C.c_int32, C.c_int32, C.c_int64, C.c_uint32, C.c_void_p,
                                      C.c_void_p, C.c_void_p]),
    "ykh_step": (C.c_int32, [_P, _I32P]),
    "ykh_num_running": (C.c_int32, [_P]),
    "ykh_num_waiting": (C.c_int32, [_P]),
    "ykh_generated": (C.c_int32, [_P, C.c_uint32, _U32P, C.c_int32, _I32P]),
    "ykh_counters": (C.c_int32, [_P, C.POINTER(C.c_int64), C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "ykh_usage": (C.c_float, [_P, C.c_int32]),
    "ykh_set_window_reclaim": (C.c_int32, [_P, C.c_int32]),
    "ykh_set_draft_shard": (C.c_int32, [_P, _P, C.c_int32, C.c_int32]),
}

_lib = None
_host = None


def _load(path: Path, protos: dict):
    if not path.exists():
        raise RuntimeError(f"{path.name} is not built; run __graft_entry__.build() (the CUDA module is required)")
    lib = C.CDLL(str(path))
    for name, (res, args) in protos.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def lib():
    global _lib
    if _lib is None:
        _lib = _load(LIB_PATH, _PROTOS)
    return _lib


def host_lib():
    global _host
    if _host is None:
        lib()
        _host = _load(HOST_LIB_PATH, _HOST_PROTOS)
    return _host


def exported_symbols() -> list[str]:
    return list(_PROTOS) + list(_HOST_PROTOS)


def last_error() -> str:
    buf = C.create_string_buffer(4096)
    lib().yk_last_error(buf, 4096)
    return buf.value.decode(errors="replace")


def check(status: int):
    if status != YK_OK:
        raise YKError(status, last_error())


def ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(C.POINTER(ctype))


def u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


def i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def bf16_bits(a) -> np.ndarray:
    """fp32 -> bf16 bit patterns (round to nearest even)."""
    u = f32(a).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def bf16_value(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def gemm_bf16_test(engine: "Engine", W_bits: np.ndarray, X_bits: np.ndarray, grid: int = 0) -> np.ndarray:
    """Y = X W^T through the tcgen05 GEMM (test hook of include/yk_testing.h)."""
    n_out, K = W_bits.shape
    m_tok = X_bits.shape[0]
    W_bits = np.ascontiguousarray(W_bits, dtype=np.uint16)
    X_bits = np.ascontiguousarray(X_bits, dtype=np.uint16)
    Y = np.zeros((m_tok, n_out), np.float32)
    check(lib().ykt_gemm_bf16(engine.h, ptr(W_bits, C.c_uint16), ptr(X_bits, C.c_uint16), n_out, K, m_tok, grid,
                              ptr(Y, C.c_float)))
    return Y


def gemm_bf16_timed(engine: "Engine", W_bits: np.ndarray, X_bits: np.ndarray, grid: int = 0, reps: int = 10):
    """(Y, ms per launch, per-CTA phase stamps [grid x 8], grid used) of the tcgen05 GEMM test hook.
    reps < 0 times -reps launches one by one, each after an L2 flush."""
    n_out, K = W_bits.shape
    m_tok = X_bits.shape[0]
    W_bits = np.ascontiguousarray(W_bits, dtype=np.uint16)
    X_bits = np.ascontiguousarray(X_bits, dtype=np.uint16)
    Y = np.zeros((m_tok, n_out), np.float32)
    ms = C.c_float()
    cap = max(4096, grid, 8 * ((n_out + 127) // 128) * ((m_tok + 255) // 256))  # >= any grid the hook uses
    st = np.zeros((cap, 8), np.uint64)
    g = C.c_int32()
    check(lib().ykt_gemm_bf16_timed(engine.h, ptr(W_bits, C.c_uint16), ptr(X_bits, C.c_uint16), n_out, K, m_tok,
                                    grid, reps, ptr(Y, C.c_float), C.byref(ms), ptr(st, C.c_uint64), C.byref(g)))
    return Y, ms.value, st[: g.value], g.value


def gemm_bf16_epi_timed(engine: "Engine", W_bits: np.ndarray, X_bits: np.ndarray, epi: int, grid: int = 0,
                        reps: int = -5, head_dim: int = 128, kv_dim: int = 1024):
    """(ms per launch, per-CTA phase stamps, grid used) of the GEMM test hook with a fused epilogue."""
    n_out, K = W_bits.shape
    m_tok = X_bits.shape[0]
    W_bits = np.ascontiguousarray(W_bits, dtype=np.uint16)
    X_bits = np.ascontiguousarray(X_bits, dtype=np.uint16)
    ms = C.c_float()
    cap = max(4096, grid, 8 * ((n_out + 127) // 128) * ((m_tok + 255) // 256))
    st = np.zeros((cap, 8), np.uint64)
    g = C.c_int32()
    check(lib().ykt_gemm_bf16_epi_timed(engine.h, ptr(W_bits, C.c_uint16), ptr(X_bits, C.c_uint16), n_out, K, m_tok,
                                        grid, reps, epi, head_dim, kv_dim, C.byref(ms), ptr(st, C.c_uint64),
                                        C.byref(g)))
    return ms.value, st[: g.value], g.value


def tp_unique_id() -> bytes:
    """A new NCCL unique id (128 bytes) for a tensor-parallel group."""
    buf = (C.c_uint8 * 128)()
    check(lib().yk_tp_unique_id(buf))
    return bytes(buf)


# ---------------------------------------------------------------------------
# Thin object wrappers.
# ---------------------------------------------------------------------------
class Engine:
    def __init__(self, device: int = 0):
        self.h = _P()
        check(lib().yk_engine_create(device, C.byref(self.h)))
        self.device = device

    def stream(self) -> int:
        s = _P()
        check(lib().yk_engine_stream(self.h, C.byref(s)))
        return s.value or 0

    def trace(self, cap: int) -> None:
        """Test hook: (re)start the launch trace with `cap` records (0 stops it)."""
        check(lib().ykt_trace_enable(self.h, cap))
        self._trace_cap = cap

    def trace_read(self) -> tuple[np.ndarray, int]:
        """Launch trace records [cap x 4] (entry, start, end ns, kind) and the launch count."""
        out = np.zeros((self._trace_cap, 4), np.uint64)
        n = C.c_uint64()
        check(lib().ykt_trace_read(self.h, ptr(out, C.c_uint64), self._trace_cap, C.byref(n)))
        return out, int(n.value)

    def tp_init(self, uid: bytes, rank: int, world: int, timeout_ms: int | None = None) -> None:
        """Join a tensor-parallel NCCL group (uid from tp_unique_id on rank 0); set-up and
        later waits on the group's work give up after timeout_ms (default 300 s)."""
        buf = (C.c_uint8 * 128).from_buffer_copy(uid)
        if timeout_ms is None:
            check(lib().yk_tp_init(self.h, buf, rank, world))
        else:
            check(lib().yk_tp_init_timeout(self.h, buf, rank, world, int(timeout_ms)))

    def sync(self):
        check(lib().yk_engine_sync(self.h))

    def wait_timeout(self, budget_ms: int) -> tuple[int, float]:
        """Test hook: a bounded device wait on a barrier nothing arrives at; returns
        (status, milliseconds the kernel waited)."""
        ms = C.c_double()
        st = lib().ykt_wait_timeout(self.h, budget_ms, C.byref(ms))
        return st, ms.value

    def tp_allreduce_timed(self, count: int, iters: int, own: bool):
        """Test hook (collective): (milliseconds per all-reduce of `count` bf16
        elements over `iters` calls back to back, phase stamps of one more call in ns
        or None); own: the group's kernel, else ncclAllReduce."""
        ms = C.c_double()
        st = (C.c_uint64 * 8)()
        check(lib().ykt_tp_allreduce_timed(self.h, int(count), int(iters), 1 if own else 0, C.byref(ms), st))
        return ms.value, ([int(x) for x in st] if own else None)

    def device_error(self) -> int:
        v = C.c_uint32()
        check(lib().yk_engine_device_error(self.h, C.byref(v)))
        return v.value

    def launches(self) -> int:
        return int(lib().yk_engine_launch_count(self.h))

    def profile(self, enable: bool):
        check(lib().yk_engine_profile(self.h, 1 if enable else 0))

    def profile_read(self, cls: int) -> dict:
        ms, b, f, n = C.c_double(), C.c_double(), C.c_double(), C.c_int64()
        check(lib().yk_engine_profile_read(self.h, cls, C.byref(ms), C.byref(b), C.byref(f), C.byref(n)))
        return {"ms": ms.value, "bytes": b.value, "flops": f.value, "launches": n.value}

    def close(self):
        if self.h:
            lib().yk_engine_destroy(self.h)
            self.h = _P()


class TensorInfo(C.Structure):
    """yk_tensor_info (include/yk.h)."""
    _fields_ = [("dtype", C.c_int32), ("dtype_name", C.c_char * 12), ("ndim", C.c_int32),
                ("shape", C.c_int64 * 8), ("data", C.c_void_p), ("nbytes", C.c_uint64)]


_NP_DTYPES = {"F32": np.float32, "F16": np.float16, "F64": np.float64, "I64": np.int64, "I32": np.int32,
              "I16": np.int16, "I8": np.int8, "U8": np.uint8, "U16": np.uint16, "U32": np.uint32,
              "U64": np.uint64, "BOOL": np.bool_, "BF16": np.uint16}  # BF16: the raw 16-bit words


def hf_tensor_id(name: str, n_layers: int) -> tuple[int, int]:
    """(tensor, layer) of a Hugging Face checkpoint name (yk_hf_tensor_id)."""
    t, l = C.c_int32(), C.c_int32()
    check(lib().yk_hf_tensor_id(name.encode(), n_layers, C.byref(t), C.byref(l)))
    return t.value, l.value


class SafeTensors:
    """A mapped .safetensors file (SafetensorsReader): names, info, raw arrays."""

    def __init__(self, path):
        self.h = _P()
        check(lib().yk_safetensors_open(str(path).encode(), C.byref(self.h)))

    def __len__(self) -> int:
        return int(lib().yk_safetensors_count(self.h))

    def names(self) -> list[str]:
        out = []
        for i in range(len(self)):
            n = C.c_char_p()
            check(lib().yk_safetensors_name(self.h, i, C.byref(n)))
            out.append(n.value.decode())
        return out

    def info(self, name: str) -> TensorInfo:
        ti = TensorInfo()
        check(lib().yk_safetensors_info(self.h, name.encode(), C.byref(ti)))
        return ti

    def array(self, name: str) -> np.ndarray:
        """A copy of the tensor's bytes as a numpy array (BF16 as uint16 words)."""
        ti = self.info(name)
        dt = np.dtype(_NP_DTYPES[ti.dtype_name.decode()])
        raw = C.string_at(ti.data, ti.nbytes) if ti.nbytes else b""
        return np.frombuffer(raw, dtype=dt).reshape(tuple(ti.shape[: ti.ndim])).copy()

    def close(self):
        if self.h:
            lib().yk_safetensors_close(self.h)
            self.h = _P()


class Model:
    def __init__(self, engine: Engine, cfg: ModelConfig, seed: int = 1, init_std: float = 0.02, tp=None):
        """tp = (rank, world): shard `rank` of a tensor-parallel target (the engine joined the group)."""
        self.engine = engine
        self.cfg = cfg
        self.h = _P()
        if tp is None:
            check(lib().yk_model_create(engine.h, C.byref(cfg), seed, init_std, C.byref(self.h)))
        else:
            check(lib().yk_model_create_tp(engine.h, C.byref(cfg), tp[0], tp[1], seed, init_std, C.byref(self.h)))
            shard = ModelConfig()
            check(lib().yk_model_get_config(self.h, C.byref(shard)))
            self.cfg = shard  # the shard's heads / FFN: the config its KV pool is created with

    def shape(self, t: int) -> tuple[int, int]:
        r, c = C.c_int64(), C.c_int64()
        check(lib().yk_model_tensor_shape(self.h, t, C.byref(r), C.byref(c)))
        return r.value, c.value

    def get(self, t: int, layer: int = 0) -> np.ndarray:
        r, c = self.shape(t)
        out = np.empty((r, c), dtype=np.float32)
        check(lib().yk_model_get_tensor(self.h, t, layer, ptr(out, C.c_float)))
        return out[0] if r == 1 else out

    def set(self, t: int, layer: int, host: np.ndarray, layout: int = LAYOUT_OUT_IN):
        a = f32(host)
        check(lib().yk_model_set_tensor(self.h, t, layer, ptr(a, C.c_float), layout))

    def load(self, t: int, layer: int, host: np.ndarray, src_dtype: int, layout: int = LAYOUT_OUT_IN):
        """yk_model_load_tensor: host holds the full stored tensor (BF16 as uint16 words)."""
        a = np.ascontiguousarray(host)
        want = {DTYPE_F32: np.float32, DTYPE_BF16: np.uint16, DTYPE_F16: np.float16}[src_dtype]
        assert a.dtype == want, (a.dtype, want)
        rows, cols = (1, a.shape[0]) if a.ndim == 1 else a.shape
        check(lib().yk_model_load_tensor(self.h, t, layer, a.ctypes.data_as(_P), src_dtype, rows, cols, layout))

    def load_safetensors(self, files, norm_offset: float = 0.0, flags: int = 0) -> int:
        arr = (_P * len(files))(*[f.h for f in files])
        n = C.c_int32()
        check(lib().yk_model_load_safetensors(self.h, arr, len(files), norm_offset, flags, C.byref(n)))
        return n.value

    def forward_split(self, pool: "KVPool", wpool: "KVPool", tokens, q_starts, ctx, block_tables: np.ndarray,
                      wblock_tables: np.ndarray, last_n: int = 0) -> int:
        """yk_forward_step_split: global layers in `pool`, windowed ones in `wpool`."""
        tok, qs, cl = u32(tokens), u32(q_starts), u32(ctx)
        bt, wbt = i32(block_tables), i32(wblock_tables)
        rows = C.c_int32()
        check(lib().yk_forward_step_split(self.h, pool.h, wpool.h, ptr(tok, C.c_uint32), len(tok),
                                          ptr(qs, C.c_uint32), ptr(cl, C.c_uint32), len(cl), ptr(bt, C.c_int32),
                                          bt.shape[1], ptr(wbt, C.c_int32), wbt.shape[1], last_n, None, 0, 0,
                                          C.byref(rows)))
        return rows.value

    def forward(self, pool: "KVPool", tokens, q_starts, ctx, block_tables: np.ndarray, last_n: int = 0) -> int:
        tok, qs, cl = u32(tokens), u32(q_starts), u32(ctx)
        bt = i32(block_tables)
        rows = C.c_int32()
        check(lib().yk_forward_step(self.h, pool.h, ptr(tok, C.c_uint32), len(tok), ptr(qs, C.c_uint32),
                                    ptr(cl, C.c_uint32), len(cl), ptr(bt, C.c_int32), bt.shape[1], last_n,
                                    C.byref(rows)))
        return rows.value

    def attention_stamps(self, cap: int = 0):
        """Test hook: cap > 0 enables per-CTA attention stamps; cap == 0 returns the
        last launch's records ([n_ctas x 8] uint64)."""
        if cap > 0:
            check(lib().ykt_attention_stamps_enable(self.h, cap))
            return None
        out = np.zeros((4096, 8), np.uint64)
        n = C.c_int32()
        check(lib().ykt_attention_stamps_read(self.h, ptr(out, C.c_uint64), 4096, C.byref(n)))
        return out[: n.value]

    def gemm_stamps(self, kind: int | None = None):
        """Test hook: kind (a GEMM trace kind; 0 disables) selects the launches that
        record per-CTA stamps; kind None returns the last one's ([n_ctas x 8] uint64)."""
        if kind is not None:
            check(lib().ykt_gemm_stamps_enable(self.h, kind))
            return None
        out = np.zeros((1024, 8), np.uint64)
        n = C.c_int32()
        check(lib().ykt_gemm_stamps_read(self.h, ptr(out, C.c_uint64), 1024, C.byref(n)))
        return out[: n.value]

    def logits(self, row0: int, rows: int) -> np.ndarray:
        out = np.empty((rows, self.cfg.vocab_size), dtype=np.float32)
        check(lib().yk_logits_copy_to_host(self.h, row0, rows, ptr(out, C.c_float)))
        return out

    def close(self):
        if self.h:
            lib().yk_model_destroy(self.h)
            self.h = _P()


POOL_ALL_LAYERS, POOL_GLOBAL_LAYERS, POOL_WINDOWED_LAYERS = 0, 1, 2


class KVPool:
    def __init__(self, engine: Engine, cfg: ModelConfig, num_blocks: int, layers: int = POOL_ALL_LAYERS):
        """layers: POOL_ALL_LAYERS, or one kind of layer (yk_kv_pool_create_layers)."""
        self.cfg = cfg
        self.h = _P()
        check(lib().yk_kv_pool_create_layers(engine.h, C.byref(cfg), num_blocks, layers, C.byref(self.h)))

    def fill_random(self, seed: int, std: float):
        check(lib().yk_kv_pool_fill_random(self.h, seed, std))

    def read_page(self, block: int, layer: int, kv: int) -> np.ndarray:
        out = np.empty((self.cfg.n_kv_heads, BLOCK_SIZE, self.cfg.head_dim), dtype=np.float32)
        check(lib().yk_kv_pool_read_page(self.h, block, layer, kv, ptr(out, C.c_float)))
        return out

    def close(self):
        if self.h:
            lib().yk_kv_pool_destroy(self.h)
            self.h = _P()


class Sampler:
    def __init__(self, engine: Engine, max_seqs: int, k: int, vocab: int):
        self.k, self.vocab = k, vocab
        self.h = _P()
        check(lib().yk_sampler_create(engine.h, max_seqs, k, vocab, C.byref(self.h)))

    def verify_probs(self, p: np.ndarray, q: np.ndarray, drafts, seed: int, step: int, seq_ids):
        B = p.shape[0]
        p, q, d, s = f32(p), f32(q), u32(drafts), u32(seq_ids)
        out = np.zeros((B, self.k + 1), dtype=np.uint32)
        cnt = np.zeros(B, dtype=np.int32)
        check(lib().yk_spec_verify_probs(self.h, B, ptr(p, C.c_float), ptr(q, C.c_float), ptr(d, C.c_uint32), seed,
                                         step, ptr(s, C.c_uint32), ptr(out, C.c_uint32), ptr(cnt, C.c_int32)))
        return out, cnt

    def sample_logits(self, dl, tl, T: float, seed: int, step: int, seq_ids):
        """dl, tl: host logits [B x k x V], [B x (k+1) x V]; both None: the logits the
        previous call uploaded (same B, from len(seq_ids)) are sampled again."""
        s = u32(seq_ids)
        B = len(s)
        if dl is None:
            pd = pt = None
        else:
            dl, tl = f32(dl), f32(tl)
            if dl.shape[0] != B or tl.shape[0] != B:
                raise ValueError("logits and seq_ids disagree on B")
            pd, pt = ptr(dl, C.c_float), ptr(tl, C.c_float)
        drafts = np.zeros((B, self.k), dtype=np.uint32)
        out = np.zeros((B, self.k + 1), dtype=np.uint32)
        cnt = np.zeros(B, dtype=np.int32)
        check(lib().yk_spec_sample_logits(self.h, B, pd, pt, T, seed, step, ptr(s, C.c_uint32),
                                          ptr(drafts, C.c_uint32), ptr(out, C.c_uint32), ptr(cnt, C.c_int32)))
        return drafts, out, cnt

    def draft_sample(self, model: Model, B: int, j: int, T: float, seed: int, step: int, seq_ids):
        s = u32(seq_ids)
        out = np.zeros(B, dtype=np.uint32)
        check(lib().yk_draft_sample(self.h, model.h, B, j, T, seed, step, ptr(s, C.c_uint32), ptr(out, C.c_uint32)))
        return out

    def verify(self, model: Model, B: int, T: float, seed: int, step: int, seq_ids, drafts):
        s, d = u32(seq_ids), u32(drafts)
        out = np.zeros((B, self.k + 1), dtype=np.uint32)
        cnt = np.zeros(B, dtype=np.int32)
        check(lib().yk_spec_verify(self.h, model.h, B, T, seed, step, ptr(s, C.c_uint32), ptr(d, C.c_uint32),
                                   ptr(out, C.c_uint32), ptr(cnt, C.c_int32)))
        return out, cnt

    def read_probs(self, b: int, j: int) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32)
        check(lib().yk_sampler_read_probs(self.h, b, j, ptr(out, C.c_float)))
        return out

    def target_probs(self, B: int, T: float) -> np.ndarray:
        """Test hook: q[B x (k+1) x V] exactly as the last sample_logits verification formed it."""
        out = np.empty((B, self.k + 1, self.vocab), dtype=np.float32)
        check(lib().ykt_sampler_target_probs(self.h, B, T, ptr(out, C.c_float)))
        return out

    def stamps(self, cap: int = 0):
        """Test hook: cap > 0 enables phase stamps; cap == 0 returns ([cap x 8] draft, [cap x 8] verify)."""
        if cap > 0:
            check(lib().ykt_sampler_stamps_enable(self.h, cap))
            self._stamps_cap = cap
            return None
        out = np.zeros((2 * self._stamps_cap, 8), np.uint64)
        check(lib().ykt_sampler_stamps_read(self.h, ptr(out, C.c_uint64), self._stamps_cap))
        return out[: self._stamps_cap], out[self._stamps_cap:]

    def close(self):
        if self.h:
            lib().yk_sampler_destroy(self.h)
            self.h = _P()


class Scheduler:
    """libyk_host.so's Scheduler (restates S/Scheduler.swift's speculative loop)."""

    def __init__(self, target: Model, tpool: KVPool, draft: Model, dpool: KVPool, sampler: Sampler, k: int,
                 temperature: float, seed: int, twpool: KVPool | None = None, dwpool: KVPool | None = None):
        """twpool / dwpool: windowed-layer pools (ykh_scheduler_create_split)."""
        self.h = _P()
        if twpool is None:
            check(host_lib().ykh_scheduler_create(target.h, tpool.h, draft.h, dpool.h, sampler.h, k, temperature, seed,
                                                  C.byref(self.h)))
        else:
            check(host_lib().ykh_scheduler_create_split(target.h, tpool.h, twpool.h, draft.h, dpool.h, dwpool.h,
                                                        sampler.h, k, temperature, seed, C.byref(self.h)))

    def submit(self, prompt, max_tokens: int, stop_token: int = -1, seq_id: int = 0, cached: bool = False):
        p = u32(prompt)
        fn = host_lib().ykh_submit_cached if cached else host_lib().ykh_submit
        check(fn(self.h, ptr(p, C.c_uint32), len(p), max_tokens, stop_token, seq_id))

    _ON_TOKENS = C.CFUNCTYPE(None, C.c_void_p, C.c_uint32, C.POINTER(C.c_uint32), C.c_int32)
    _ON_DONE = C.CFUNCTYPE(None, C.c_void_p, C.c_uint32, C.c_int32)

    def set_window_reclaim(self, on: bool):
        check(host_lib().ykh_set_window_reclaim(self.h, 1 if on else 0))

    def set_draft_shard(self, engine: "Engine", rank: int, world: int):
        """Sequence-sharded drafting across a tensor-parallel group (ykh_set_draft_shard)."""
        check(host_lib().ykh_set_draft_shard(self.h, engine.h, rank, world))

    def submit_stream(self, prompt, max_tokens: int, on_tokens=None, on_done=None, stop_token: int = -1,
                      seq_id: int = 0):
        """ykh_submit_stream: on_tokens(seq_id, list_of_token_ids) per emitted run,
        on_done(seq_id, n_generated) once; called inside step()."""
        p = u32(prompt)
        ct = self._ON_TOKENS(lambda _u, sid, toks, n: on_tokens(int(sid), [toks[i] for i in range(n)])) \
            if on_tokens else C.cast(None, self._ON_TOKENS)
        cd = self._ON_DONE(lambda _u, sid, n: on_done(int(sid), int(n))) if on_done else C.cast(None, self._ON_DONE)
        if not hasattr(self, "_callbacks"):
            self._callbacks = []
        self._callbacks.append((ct, cd))  # the C side keeps the pointers until the request is done
        check(host_lib().ykh_submit_stream(self.h, ptr(p, C.c_uint32), len(p), max_tokens, stop_token, seq_id,
                                           C.cast(ct, C.c_void_p), C.cast(cd, C.c_void_p), None))

    def step(self) -> int:
        e = C.c_int32()
        check(host_lib().ykh_step(self.h, C.byref(e)))
        return e.value

    def running(self) -> int:
        return host_lib().ykh_num_running(self.h)

    def waiting(self) -> int:
        return host_lib().ykh_num_waiting(self.h)

    def generated(self, seq_id: int) -> list[int]:
        n = C.c_int32()
        check(host_lib().ykh_generated(self.h, seq_id, None, 0, C.byref(n)))
        out = np.zeros(max(n.value, 1), dtype=np.uint32)
        check(host_lib().ykh_generated(self.h, seq_id, ptr(out, C.c_uint32), n.value, C.byref(n)))
        return out[: n.value].tolist()

    def counters(self) -> tuple[int, int, int]:
        a, b, c = C.c_int64(), C.c_int64(), C.c_int64()
        check(host_lib().ykh_counters(self.h, C.byref(a), C.byref(b), C.byref(c)))
        return a.value, b.value, c.value

    def usage(self, draft: bool = False) -> float:
        return float(host_lib().ykh_usage(self.h, 1 if draft else 0))

    def usage_windowed(self, draft: bool = False) -> float:
        return float(host_lib().ykh_usage_windowed(self.h, 1 if draft else 0))

    def close(self):
        if self.h:
            host_lib().ykh_scheduler_destroy(self.h)
            self.h = _P()
