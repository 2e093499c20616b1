"""ctypes binding of the CPU oracle (oracle/liboracle.so) -- test infrastructure.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use this;
the CUDA module never does.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
ORACLE_DIR = ROOT / "oracle"
ORACLE_LIB = ORACLE_DIR / "liboracle.so"

SLOT_DRAFT, SLOT_ACCEPT, SLOT_RESAMPLE, SLOT_BONUS = 0, 1, 2, 3

_F = C.POINTER(C.c_float)
_U = C.POINTER(C.c_uint32)
_I = C.POINTER(C.c_int32)


class OrcCfg(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int32), ("d_model", C.c_int32), ("n_layers", C.c_int32), ("n_heads", C.c_int32),
        ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn_dim", C.c_int32),
        ("rope_theta", C.c_float), ("rms_eps", C.c_float), ("attn_cap", C.c_float), ("final_cap", C.c_float),
        ("window", C.c_int32), ("window_layer_parity", C.c_int32), ("act", C.c_int32), ("ref_compat", C.c_int32),
        ("emulate_bf16", C.c_int32), ("block_size", C.c_int32),
    ]


class OrcWeights(C.Structure):
    _fields_ = [("embed", _F), ("wq", C.POINTER(_F)), ("wk", C.POINTER(_F)), ("wv", C.POINTER(_F)),
                ("wo", C.POINTER(_F)), ("wg", C.POINTER(_F)), ("wu", C.POINTER(_F)), ("wd", C.POINTER(_F)),
                ("n1", C.POINTER(_F)), ("n2", C.POINTER(_F)), ("final_norm", _F), ("lm_head", _F)]


_lib = None


def build_oracle():
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not ORACLE_LIB.exists():
            build_oracle()
        L = C.CDLL(str(ORACLE_LIB))
        L.orc_philox4x32_10.argtypes = [_U, _U, _U]
        L.orc_uniform.restype = C.c_float
        L.orc_uniform.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]
        L.orc_softmax.argtypes = [_F, C.c_int64, C.c_float, _F]
        L.orc_sample_from_probs.restype = C.c_uint32
        L.orc_sample_from_probs.argtypes = [_F, C.c_int64, C.c_float]
        L.orc_verify_token.restype = C.c_int
        L.orc_verify_token.argtypes = [C.c_uint32, _F, _F, C.c_int64, C.c_float, C.c_float, _U]
        L.orc_verify_sequence_probs.restype = C.c_int
        L.orc_verify_sequence_probs.argtypes = [_U, C.c_int, _F, _F, C.c_int64, C.c_uint64, C.c_uint32, C.c_uint32, _U]
        L.orc_verify_sequence_logits.restype = C.c_int
        L.orc_verify_sequence_logits.argtypes = [_U, C.c_int, _F, _F, C.c_int64, C.c_float, C.c_uint64, C.c_uint32,
                                                 C.c_uint32, _U]
        L.orc_draft_sample.restype = C.c_uint32
        L.orc_draft_sample.argtypes = [_F, C.c_int64, C.c_float, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, _F]
        L.orc_argmax.restype = C.c_uint32
        L.orc_argmax.argtypes = [_F, C.c_int64]
        L.orc_verify_batch_probs.argtypes = [C.c_int, C.c_int, C.c_int64, _U, _F, _F, C.c_uint64, C.c_uint32, _U,
                                             C.c_int, _U, _I]
        L.orc_spec_sample_batch.argtypes = [C.c_int, C.c_int, C.c_int64, _F, _F, C.c_float, C.c_uint64, C.c_uint32,
                                            _U, C.c_int, _U, _U, _I]
        L.orc_pool_floats.restype = C.c_size_t
        L.orc_pool_floats.argtypes = [C.POINTER(OrcCfg), C.c_int32]
        L.orc_forward_step.restype = C.c_int
        L.orc_forward_step.argtypes = [C.POINTER(OrcCfg), C.POINTER(OrcWeights), _F, C.c_int32, _U, C.c_int32, _U, _U,
                                       C.c_int32, _I, C.c_int32, C.c_int32, C.c_int, _F]
        L.orc_bf16_round.restype = C.c_float
        L.orc_bf16_round.argtypes = [C.c_float]
        L.orc_f16_to_f32.restype = None
        L.orc_f16_to_f32.argtypes = [C.POINTER(C.c_uint16), C.c_size_t, _F]
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(C.POINTER(t))


def f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def u32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


def philox(ctr, key):
    c, k, o = u32(ctr), u32(key), np.zeros(4, np.uint32)
    lib().orc_philox4x32_10(_p(c, C.c_uint32), _p(k, C.c_uint32), _p(o, C.c_uint32))
    return [int(x) for x in o]


def uniform(seed, step, seq, pos, slot) -> float:
    return float(lib().orc_uniform(seed, step, seq, pos, slot))


def softmax(logits, T=1.0):
    x = f32(logits)
    out = np.empty_like(x)
    lib().orc_softmax(_p(x, C.c_float), x.size, T, _p(out, C.c_float))
    return out


def sample_from_probs(probs, r) -> int:
    x = f32(probs)
    return int(lib().orc_sample_from_probs(_p(x, C.c_float), x.size, r))


def verify_token(d, p, q, ra, rr):
    p, q = f32(p), f32(q)
    nt = np.zeros(1, np.uint32)
    acc = lib().orc_verify_token(d, _p(p, C.c_float), _p(q, C.c_float), p.size, ra, rr, _p(nt, C.c_uint32))
    return bool(acc), int(nt[0])


def verify_sequence_probs(drafts, p, q, seed, step, seq):
    d, p, q = u32(drafts), f32(p), f32(q)
    k, V = p.shape
    out = np.zeros(k + 1, np.uint32)
    n = lib().orc_verify_sequence_probs(_p(d, C.c_uint32), k, _p(p, C.c_float), _p(q, C.c_float), V, seed, step, seq,
                                        _p(out, C.c_uint32))
    return out[:n].tolist()


def verify_batch_probs(drafts, p, q, seed, step, seq_ids, nthreads=8):
    d, p, q, s = u32(drafts), f32(p), f32(q), u32(seq_ids)
    B, k, V = p.shape
    out = np.zeros((B, k + 1), np.uint32)
    cnt = np.zeros(B, np.int32)
    lib().orc_verify_batch_probs(B, k, V, _p(d, C.c_uint32), _p(p, C.c_float), _p(q, C.c_float), seed, step,
                                 _p(s, C.c_uint32), nthreads, _p(out, C.c_uint32), _p(cnt, C.c_int32))
    return out, cnt


def spec_sample_batch(dl, tl, T, seed, step, seq_ids, nthreads=8):
    dl, tl, s = f32(dl), f32(tl), u32(seq_ids)
    B, k, V = dl.shape
    drafts = np.zeros((B, k), np.uint32)
    out = np.zeros((B, k + 1), np.uint32)
    cnt = np.zeros(B, np.int32)
    lib().orc_spec_sample_batch(B, k, V, _p(dl, C.c_float), _p(tl, C.c_float), T, seed, step, _p(s, C.c_uint32),
                                nthreads, _p(drafts, C.c_uint32), _p(out, C.c_uint32), _p(cnt, C.c_int32))
    return drafts, out, cnt


def draft_sample(logits, T, seed, step, seq, j):
    x = f32(logits)
    p = np.empty_like(x)
    tok = lib().orc_draft_sample(_p(x, C.c_float), x.size, T, seed, step, seq, j, _p(p, C.c_float))
    return int(tok), p


def bf16_round(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


class OracleModel:
    """fp32 weights + a paged pool for orc_forward_step."""

    def __init__(self, cfg: dict, weights: dict, num_blocks: int, emulate_bf16: bool = False, nthreads: int = 8):
        self.c = OrcCfg()
        for k in ("vocab_size", "d_model", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn_dim", "rope_theta",
                  "rms_eps", "attn_cap", "final_cap", "window", "window_layer_parity", "act", "ref_compat"):
            setattr(self.c, k, cfg[k])
        self.c.emulate_bf16 = 1 if emulate_bf16 else 0
        self.c.block_size = 16
        self.cfg = cfg
        self.nthreads = nthreads
        self.num_blocks = num_blocks
        self.pool = np.zeros(lib().orc_pool_floats(C.byref(self.c), num_blocks), dtype=np.float32)
        self._keep = {k: (f32(v) if not isinstance(v, list) else [f32(x) for x in v]) for k, v in weights.items()}
        L = cfg["n_layers"]
        w = OrcWeights()
        w.embed = _p(self._keep["embed"], C.c_float)
        w.final_norm = _p(self._keep["final_norm"], C.c_float)
        w.lm_head = _p(self._keep["lm_head"], C.c_float)
        self._arrs = []
        for name in ("wq", "wk", "wv", "wo", "wg", "wu", "wd", "n1", "n2"):
            arr = (_F * L)(*[_p(x, C.c_float) for x in self._keep[name]])
            self._arrs.append(arr)
            setattr(w, name, C.cast(arr, C.POINTER(_F)))
        self.w = w

    def forward(self, tokens, q_starts, ctx, block_tables, last_n=0):
        tok, qs, cl = u32(tokens), u32(q_starts), u32(ctx)
        bt = np.ascontiguousarray(block_tables, dtype=np.int32)
        B = len(cl)
        n = np.diff(qs)
        rows = int(sum(min(last_n, x) if last_n > 0 else x for x in n))
        out = np.zeros((rows, self.cfg["vocab_size"]), np.float32)
        rc = lib().orc_forward_step(C.byref(self.c), C.byref(self.w), _p(self.pool, C.c_float), self.num_blocks,
                                    _p(tok, C.c_uint32), len(tok), _p(qs, C.c_uint32), _p(cl, C.c_uint32), B,
                                    _p(bt, C.c_int32), bt.shape[1], last_n, self.nthreads, _p(out, C.c_float))
        if rc != 0:
            raise ValueError("oracle forward rejected its arguments")
        return out


def f16_to_f32(h):
    """The reference's F16 checkpoint conversion (uint16 words -> fp32)."""
    a = np.ascontiguousarray(np.asarray(h, dtype=np.uint16))
    out = np.empty(a.shape, np.float32)
    lib().orc_f16_to_f32(_p(a, C.c_uint16), a.size, _p(out, C.c_float))
    return out
