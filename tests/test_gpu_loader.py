"""Checkpoint loading through the C-ABI on the device: yk_model_load_tensor
(ModelLoader.loadLinearLayer, S/ModelLoader.swift:9-72, plus BF16 sources and
the [out x in] layout) and yk_model_load_safetensors (Hugging Face names).
Every loaded value is compared bit for bit with the oracle's conversions."""
from __future__ import annotations

import numpy as np
import pytest

import oracle_ffi as oracle
from helpers import TINY, PageTables, forward_pair, gpu_model, oracle_twin
from st_writer import bf16_words, write_safetensors
from test_safetensors import unpermute_rope_half
from yanaiengine_b200 import abi

pytestmark = pytest.mark.gpu

PER_LAYER = (abi.T_WQ, abi.T_WK, abi.T_WV, abi.T_WO, abi.T_WGATE, abi.T_WUP, abi.T_WDOWN, abi.T_NORM1, abi.T_NORM2)


def _source(rng, shape, src_dtype):
    """(stored array, its exact fp32 values)."""
    v = rng.standard_normal(shape).astype(np.float32)
    if src_dtype == abi.DTYPE_F32:
        return v, v
    if src_dtype == abi.DTYPE_BF16:
        w = bf16_words(v)
        return w, (w.astype(np.uint32) << 16).view(np.float32)
    h = v.astype(np.float16)
    return h, oracle.f16_to_f32(h.view(np.uint16))


def _expected(vals: np.ndarray, t: int, model_dtype: int) -> np.ndarray:
    if model_dtype == abi.DTYPE_F32 or t in (abi.T_NORM1, abi.T_NORM2, abi.T_FINAL_NORM):
        return vals  # norms are fp32 in every model
    return np.vectorize(oracle.lib().orc_bf16_round, otypes=[np.float32])(vals)


@pytest.mark.parametrize("model_dtype", [abi.DTYPE_BF16, abi.DTYPE_F32])
@pytest.mark.parametrize("src_dtype", [abi.DTYPE_F32, abi.DTYPE_BF16, abi.DTYPE_F16])
@pytest.mark.parametrize("layout", [abi.LAYOUT_OUT_IN, abi.LAYOUT_IN_OUT])
def test_load_tensor_conversions_and_layouts(engine, model_dtype, src_dtype, layout):
    m, pool = gpu_model(engine, TINY, model_dtype, seed=5, num_blocks=4)
    rng = np.random.default_rng(10 * model_dtype + src_dtype + 100 * layout)
    try:
        for t in (abi.T_EMBED, abi.T_WQ, abi.T_WK, abi.T_WV, abi.T_WO, abi.T_WGATE, abi.T_WUP, abi.T_WDOWN,
                  abi.T_NORM1, abi.T_FINAL_NORM, abi.T_LM_HEAD):
            layer = 1 if t in PER_LAYER else 0
            rows, cols = m.shape(t)
            stored, vals = _source(rng, (rows, cols), src_dtype)
            if layout == abi.LAYOUT_IN_OUT:  # the reference's [in x out]
                stored, vals = np.ascontiguousarray(stored.T), np.ascontiguousarray(vals.T)
            m.load(t, layer, stored if rows > 1 or layout == abi.LAYOUT_IN_OUT else stored[0], src_dtype, layout)
            want = _expected(vals if layout == abi.LAYOUT_OUT_IN else vals.T, t, model_dtype)
            got = m.get(t, layer).reshape(rows, cols)
            assert (got.view(np.uint32) == want.reshape(rows, cols).view(np.uint32)).all(), (t, layer)
        # neighbours of the fused / interleaved tensors are untouched by a later load
        before = m.get(abi.T_WUP, 1)
        stored, vals = _source(rng, m.shape(abi.T_WGATE), src_dtype)
        if layout == abi.LAYOUT_IN_OUT:
            stored = np.ascontiguousarray(stored.T)
        m.load(abi.T_WGATE, 1, stored, src_dtype, layout)
        assert (m.get(abi.T_WUP, 1) == before).all()
        # shape checks: the transposed shape of a non-square tensor is refused
        r, c = m.shape(abi.T_WGATE)
        with pytest.raises(abi.YKError) as ei:
            m.load(abi.T_WGATE, 0, np.zeros((c, r) if layout == abi.LAYOUT_OUT_IN else (r, c), np.float32),
                   abi.DTYPE_F32, layout)
        assert ei.value.status == 1 and "expected" in str(ei.value)
        assert engine.device_error() == 0
    finally:
        pool.close()
        m.close()


@pytest.mark.parametrize("model_dtype", [abi.DTYPE_F32, abi.DTYPE_BF16])
def test_f16_every_bit_pattern(engine, model_dtype):
    """All 65536 half patterns through the device conversion equal the reference's
    bit-level conversion (then bf16 rounding for a bf16 model); nan stays nan."""
    m, pool = gpu_model(engine, TINY, model_dtype, seed=6, num_blocks=4)
    try:
        rows, cols = m.shape(abi.T_EMBED)
        h = (np.arange(rows * cols, dtype=np.uint32) % (1 << 16)).astype(np.uint16)
        m.load(abi.T_EMBED, 0, h.view(np.float16).reshape(rows, cols), abi.DTYPE_F16)
        got = m.get(abi.T_EMBED).ravel()
        want = _expected(oracle.f16_to_f32(h), abi.T_EMBED, model_dtype)
        nan = np.isnan(want)
        assert (np.isnan(got) == nan).all()
        assert (got[~nan].view(np.uint32) == want[~nan].view(np.uint32)).all()
    finally:
        pool.close()
        m.close()


def _hf_checkpoint(rng, cfg, tmp_path, dtype="BF16", tied=True, split=2, extra=None, drop=None):
    """A Hugging Face Llama-named checkpoint of cfg over `split` files (Q/K rows
    in rotate-half order); returns the paths and the stored arrays by name."""
    d, dh, L = cfg["d_model"], cfg["head_dim"], cfg["n_layers"]
    qd, kvd, F, V = cfg["n_heads"] * dh, cfg["n_kv_heads"] * dh, cfg["ffn_dim"], cfg["vocab_size"]
    shapes = {"model.embed_tokens.weight": (V, d), "model.norm.weight": (d,)}
    if not tied:
        shapes["lm_head.weight"] = (V, d)
    for l in range(L):
        p = f"model.layers.{l}."
        shapes.update({p + "self_attn.q_proj.weight": (qd, d), p + "self_attn.k_proj.weight": (kvd, d),
                       p + "self_attn.v_proj.weight": (kvd, d), p + "self_attn.o_proj.weight": (d, qd),
                       p + "mlp.gate_proj.weight": (F, d), p + "mlp.up_proj.weight": (F, d),
                       p + "mlp.down_proj.weight": (d, F), p + "input_layernorm.weight": (d,),
                       p + "post_attention_layernorm.weight": (d,)})
    shapes.update(extra or {})
    for k in drop or ():
        shapes.pop(k)
    arrays = {}
    for name, shp in shapes.items():
        scale = 0.02 if len(shp) == 2 else 1.0
        v = (1.0 + 0.1 * rng.standard_normal(shp) if len(shp) == 1 else scale * rng.standard_normal(shp))
        arrays[name] = bf16_words(v) if dtype == "BF16" else v.astype(np.float32)
    names = sorted(arrays)
    paths = []
    for i in range(split):
        part = {n: (dtype, arrays[n]) for n in names[i::split]}
        paths.append(tmp_path / f"model-{i + 1:05d}-of-{split:05d}.safetensors")
        write_safetensors(paths[-1], part, metadata={"format": "pt"})
    return paths, arrays


def _f32(a):
    return (a.astype(np.uint32) << 16).view(np.float32) if a.dtype == np.uint16 else a


def test_safetensors_checkpoint_loads_and_runs(engine, tmp_path):
    """A two-file bf16 checkpoint with a tied LM head: every tensor lands bit-exact
    (Q/K rows mapped out of rotate-half order), then a ragged verify step of the
    loaded model matches the oracle holding the same weights."""
    rng = np.random.default_rng(3)
    paths, arrays = _hf_checkpoint(rng, TINY, tmp_path)
    m, pool = gpu_model(engine, TINY, abi.DTYPE_BF16, seed=7, num_blocks=16)
    files = [abi.SafeTensors(p) for p in paths]
    try:
        n = m.load_safetensors(files, flags=abi.LOAD_ROPE_HALF)
        L = TINY["n_layers"]
        assert n == 3 + 9 * L
        dh = TINY["head_dim"]
        assert (m.get(abi.T_EMBED) == _f32(arrays["model.embed_tokens.weight"])).all()
        assert (m.get(abi.T_LM_HEAD) == _f32(arrays["model.embed_tokens.weight"])).all()  # tied
        assert (m.get(abi.T_FINAL_NORM) == _f32(arrays["model.norm.weight"])).all()
        for l in range(L):
            p = f"model.layers.{l}."
            for t, name, rope in ((abi.T_WQ, "self_attn.q_proj.weight", True),
                                  (abi.T_WK, "self_attn.k_proj.weight", True),
                                  (abi.T_WV, "self_attn.v_proj.weight", False),
                                  (abi.T_WO, "self_attn.o_proj.weight", False),
                                  (abi.T_WGATE, "mlp.gate_proj.weight", False),
                                  (abi.T_WUP, "mlp.up_proj.weight", False),
                                  (abi.T_WDOWN, "mlp.down_proj.weight", False),
                                  (abi.T_NORM1, "input_layernorm.weight", False),
                                  (abi.T_NORM2, "post_attention_layernorm.weight", False)):
                want = _f32(arrays[p + name])
                if rope:
                    want = unpermute_rope_half(want, dh)
                assert (m.get(t, l) == want).all(), (l, name)
        orc = oracle_twin(oracle, m, TINY, 16, emulate_bf16=True, nthreads=4)
        pt = PageTables(16)
        g, o = forward_pair(m, pool, orc, pt, [(0, rng.integers(0, 512, 19).tolist(), 0),
                                               (1, rng.integers(0, 512, 5).tolist(), 0)])
        err = np.abs(g - o).max() / np.abs(o).max()
        assert err < 2e-2, err
        # without the flag the stored row order is kept
        m.load_safetensors(files)
        assert (m.get(abi.T_WQ, 0) == _f32(arrays["model.layers.0.self_attn.q_proj.weight"])).all()
        # Gemma-style gains stored as gain - 1
        m.load_safetensors(files, norm_offset=1.0)
        assert np.array_equal(m.get(abi.T_NORM2, 1),
                              _f32(arrays["model.layers.1.post_attention_layernorm.weight"]) + np.float32(1.0))
        assert engine.device_error() == 0
    finally:
        for f in files:
            f.close()
        pool.close()
        m.close()


def test_safetensors_checkpoint_errors(engine, tmp_path):
    rng = np.random.default_rng(4)
    m, pool = gpu_model(engine, TINY, abi.DTYPE_F32, seed=8, num_blocks=4)
    try:
        def load(**kw):
            sub = tmp_path / f"c{len(list(tmp_path.iterdir()))}"
            sub.mkdir()
            paths, _ = _hf_checkpoint(rng, TINY, sub, dtype="F32", **kw)
            files = [abi.SafeTensors(p) for p in paths]
            try:
                with pytest.raises(abi.YKError) as ei:
                    m.load_safetensors(files)
                return ei.value
            finally:
                for f in files:
                    f.close()

        e = load(drop=["model.layers.1.mlp.up_proj.weight"])
        assert e.status == 1 and "lacks tensor" in str(e)
        e = load(extra={"model.layers.0.pre_feedforward_layernorm.weight": (TINY["d_model"],)})
        assert e.status == 7 and "pre_feedforward_layernorm" in str(e)
        e = load(extra={"model.layers.0.self_attn.q_proj.weight": (TINY["d_model"], TINY["d_model"] + 8)})
        assert e.status == 1 and "q_proj" in str(e) and "expected" in str(e)
        # one tensor in two files
        sub = tmp_path / "dup"
        sub.mkdir()
        paths, arrays = _hf_checkpoint(rng, TINY, sub, dtype="F32", split=1)
        write_safetensors(sub / "extra.safetensors", {"model.norm.weight": ("F32", arrays["model.norm.weight"])})
        files = [abi.SafeTensors(p) for p in (*paths, sub / "extra.safetensors")]
        try:
            with pytest.raises(abi.YKError) as ei:
                m.load_safetensors(files)
            assert ei.value.status == 1 and "more than one file" in str(ei.value)
        finally:
            for f in files:
                f.close()
        # an integer weight
        sub = tmp_path / "int"
        sub.mkdir()
        paths, arrays = _hf_checkpoint(rng, TINY, sub, dtype="F32", split=1, drop=["model.norm.weight"])
        write_safetensors(sub / "n.safetensors",
                          {"model.norm.weight": ("I32", np.ones(TINY["d_model"], np.int32))})
        files = [abi.SafeTensors(p) for p in (*paths, sub / "n.safetensors")]
        try:
            with pytest.raises(abi.YKError) as ei:
                m.load_safetensors(files)
            assert ei.value.status == 7 and "I32" in str(ei.value)
        finally:
            for f in files:
                f.close()
        assert engine.device_error() == 0
    finally:
        pool.close()
        m.close()
