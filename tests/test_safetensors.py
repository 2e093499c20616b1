"""Checkpoint reader (yk_safetensors_*, the SafetensorsReader of
S/SafetensorsReader.swift:18-128) and the oracle's F16 conversion
(S/ModelLoader.swift:75-100).  CPU only: the reader touches no device."""
from __future__ import annotations

import json

import numpy as np
import pytest

import oracle_ffi as oracle
from st_writer import bf16_words, header_and_data, write_raw, write_safetensors
from yanaiengine_b200 import abi


def test_oracle_f16_conversion_matches_ieee():
    """The restated bit-level conversion equals IEEE half -> single on all 65536
    patterns (signed zeros, subnormals, inf, nan payloads)."""
    h = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    got = oracle.f16_to_f32(h).view(np.uint32)
    want = h.view(np.float16).astype(np.float32).view(np.uint32)
    assert (got == want).all()


def test_reader_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    t = {
        "model.layers.0.self_attn.q_proj.weight": ("BF16", bf16_words(rng.standard_normal((8, 4)))),
        "a.f32": ("F32", rng.standard_normal((3, 5)).astype(np.float32)),
        "b.f16": ("F16", rng.standard_normal(7).astype(np.float16)),
        "c.i8": ("I8", rng.integers(-128, 127, (2, 2, 2)).astype(np.int8)),
        "d.scalar": ("F32", np.array(1.5, np.float32)),
        "e.empty": ("F32", np.zeros((0, 4), np.float32)),
        "café \U0001F600": ("I64", np.arange(3, dtype=np.int64)),
    }
    path = tmp_path / "m.safetensors"
    write_safetensors(path, t, metadata={"format": "pt"})
    st = abi.SafeTensors(path)
    try:
        assert len(st) == len(t)
        assert st.names() == sorted(t)  # name order, __metadata__ skipped
        codes = {"F32": abi.DTYPE_F32, "BF16": abi.DTYPE_BF16, "F16": abi.DTYPE_F16}
        for name, (dt, arr) in t.items():
            ti = st.info(name)
            assert ti.dtype_name.decode() == dt
            assert ti.dtype == codes.get(dt, -1)
            assert tuple(ti.shape[: ti.ndim]) == arr.shape
            assert ti.nbytes == arr.nbytes
            got = st.array(name)
            assert got.dtype == arr.dtype and got.shape == arr.shape
            assert got.tobytes() == arr.tobytes()
        with pytest.raises(abi.YKError) as ei:
            st.info("absent")
        assert ei.value.status == 1 and "not found" in str(ei.value)
    finally:
        st.close()


def _expect_invalid(path, what: str):
    with pytest.raises(abi.YKError) as ei:
        abi.SafeTensors(path)
    assert ei.value.status == 1, ei.value
    assert what in str(ei.value), str(ei.value)


def test_reader_rejects_malformed_files(tmp_path):
    arr = np.arange(6, dtype=np.float32).reshape(2, 3)
    good_hdr, data = header_and_data({"w": ("F32", arr)})
    p = tmp_path / "bad.safetensors"

    def write(hdr, payload=data, length=None):
        write_raw(p, json.dumps(hdr).encode() if isinstance(hdr, dict) else hdr, payload, length)

    p.write_bytes(b"\x01\x02")
    _expect_invalid(p, "shorter than")
    write(good_hdr, length=1 << 40)
    _expect_invalid(p, "header length")
    write(good_hdr, length=0)
    _expect_invalid(p, "header length")
    write(b'{"w": {"dtype": "F32", "shape": [2, 3], "data_offsets": [0, 24]')  # unterminated
    _expect_invalid(p, "not a JSON object")
    write(b"[1, 2]")
    _expect_invalid(p, "not a JSON object")
    write(b"[" * 100 + b"]" * 100)  # nesting bomb
    _expect_invalid(p, "not a JSON object")
    write({"w": {"dtype": "F32", "shape": [2, 3], "data_offsets": [0, 48]}})
    _expect_invalid(p, "outside the data block")
    write({"w": {"dtype": "F32", "shape": [2, 3], "data_offsets": [8, 4]}})
    _expect_invalid(p, "outside the data block")
    write({"w": {"dtype": "F32", "shape": [2, 2], "data_offsets": [0, 24]}})
    _expect_invalid(p, "does not match its shape")
    write({"w": {"dtype": "F32", "shape": [2, -3], "data_offsets": [0, 24]}})
    _expect_invalid(p, "bad shape")
    write({"w": {"dtype": "Q4", "shape": [2, 3], "data_offsets": [0, 24]}})
    _expect_invalid(p, "unknown dtype")
    write({"w": {"dtype": "F32", "shape": [2, 3]}})
    _expect_invalid(p, "lacks dtype")
    write({"w": {"dtype": "F32", "shape": [1] * 9, "data_offsets": [0, 4]}})
    _expect_invalid(p, "more than 8 dimensions")
    write({"w": {"dtype": "F32", "shape": [1 << 40, 1 << 40], "data_offsets": [0, 24]}})
    _expect_invalid(p, "too large")
    write(b'{"w": {"dtype": "F32", "shape": [2, 3], "data_offsets": [0, 24]}, '
          b'"w": {"dtype": "F32", "shape": [2, 3], "data_offsets": [0, 24]}}')
    _expect_invalid(p, "duplicate")
    with pytest.raises(abi.YKError):
        abi.SafeTensors(tmp_path / "missing.safetensors")


def unpermute_rope_half(w: np.ndarray, head_dim: int) -> np.ndarray:
    """Rows of a rotate-half ordered Q/K weight in interleaved-pair order: row
    2i + j of each head comes from stored row j * head_dim / 2 + i (the row map
    yk_model_load_safetensors applies under YK_LOAD_ROPE_HALF)."""
    rows = w.shape[0]
    h, r = np.divmod(np.arange(rows), head_dim)
    src = h * head_dim + (r & 1) * (head_dim // 2) + (r >> 1)
    return w[src]


def test_rope_half_row_map_preserves_attention_scores():
    """Rotate-half RoPE on rotate-half ordered weights (Hugging Face Llama) gives
    the same q.k scores as the interleaved-pair RoPE (S/gemm.metal:674-682) on
    the rows the loader maps them to."""
    rng = np.random.default_rng(1)
    dh, d, heads, theta = 64, 96, 2, 10000.0
    wq, wk = rng.standard_normal((heads * dh, d)), rng.standard_normal((heads * dh, d))
    x = rng.standard_normal((5, d))
    pos = np.array([0, 3, 17, 100, 2047])
    ang = pos[:, None] / theta ** (np.arange(dh // 2) * 2.0 / dh)[None, :]
    cos, sin = np.cos(ang), np.sin(ang)

    def rope_half(v):  # v: [T, dh]
        a, b = v[:, : dh // 2], v[:, dh // 2:]
        return np.concatenate([a * cos - b * sin, b * cos + a * sin], axis=1)

    def rope_pairs(v):
        a, b = v[:, 0::2], v[:, 1::2]
        out = np.empty_like(v)
        out[:, 0::2], out[:, 1::2] = a * cos - b * sin, a * sin + b * cos
        return out

    q_h, k_h = x @ wq.T, x @ wk.T
    q_i, k_i = x @ unpermute_rope_half(wq, dh).T, x @ unpermute_rope_half(wk, dh).T
    for h in range(heads):
        s = slice(h * dh, (h + 1) * dh)
        ref = rope_half(q_h[:, s]) @ rope_half(k_h[:, s]).T
        got = rope_pairs(q_i[:, s]) @ rope_pairs(k_i[:, s]).T
        np.testing.assert_allclose(got, ref, rtol=1e-10, atol=1e-9)


def test_hf_name_mapping():
    """The checkpoint-name map of yk_model_load_safetensors (no device needed)."""
    L = 4
    cases = {
        "model.embed_tokens.weight": (abi.T_EMBED, 0), "model.norm.weight": (abi.T_FINAL_NORM, 0),
        "lm_head.weight": (abi.T_LM_HEAD, 0),
        "model.layers.0.self_attn.q_proj.weight": (abi.T_WQ, 0), "model.layers.3.self_attn.k_proj.weight": (abi.T_WK, 3),
        "model.layers.1.self_attn.v_proj.weight": (abi.T_WV, 1), "model.layers.2.self_attn.o_proj.weight": (abi.T_WO, 2),
        "model.layers.0.mlp.gate_proj.weight": (abi.T_WGATE, 0), "model.layers.0.mlp.up_proj.weight": (abi.T_WUP, 0),
        "model.layers.3.mlp.down_proj.weight": (abi.T_WDOWN, 3),
        "model.layers.2.input_layernorm.weight": (abi.T_NORM1, 2),
        "model.layers.2.post_attention_layernorm.weight": (abi.T_NORM2, 2),
    }
    for name, want in cases.items():
        assert abi.hf_tensor_id(name, L) == want, name
    for bad in ("model.layers.4.mlp.up_proj.weight",           # layer past the model
                "model.layers.x.mlp.up_proj.weight", "model.layers..mlp.up_proj.weight",
                "model.layers.03.mlp.up_proj.weight", "model.layers.00.mlp.up_proj.weight",  # one name per slot
                "model.layers.+3.mlp.up_proj.weight", "model.layers.-0.mlp.up_proj.weight",
                "model.layers.0.pre_feedforward_layernorm.weight",  # Gemma-2 norm: no slot here
                "model.layers.0.self_attn.q_proj.bias", "model.rotary_emb.inv_freq", "lm_head", ""):
        with pytest.raises(abi.YKError) as ei:
            abi.hf_tensor_id(bad, L)
        assert ei.value.status == 1


# ---------------------------------------------------------------------------
# Property tests: the header parser faces untrusted files.
# ---------------------------------------------------------------------------
from hypothesis import HealthCheck, given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

_DT = {"F32": np.float32, "F16": np.float16, "I8": np.int8, "U8": np.uint8, "I32": np.int32, "I64": np.int64,
       "F64": np.float64, "BF16": np.uint16}


@settings(max_examples=60, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(st.dictionaries(st.text(min_size=1, max_size=12), st.tuples(st.sampled_from(sorted(_DT)),
                       st.lists(st.integers(0, 5), min_size=0, max_size=3)), min_size=0, max_size=6))
def test_reader_round_trip_property(tmp_path_factory, spec):
    """Any set of tensors (names with any characters, any dtype, shapes with zeros)
    reads back with the same names, dtypes, shapes and bytes."""
    rng = np.random.default_rng(0)
    tensors = {}
    for name, (dt, shape) in spec.items():
        if name == "__metadata__":
            continue
        a = (rng.integers(0, 100, shape) if np.issubdtype(_DT[dt], np.integer)
             else rng.standard_normal(shape)).astype(_DT[dt])
        tensors[name] = (dt, a)
    path = tmp_path_factory.mktemp("st") / "p.safetensors"
    write_safetensors(path, tensors)
    if any("\x00" in n for n in tensors):  # C strings cannot carry the name: refused
        with pytest.raises(abi.YKError) as ei:
            abi.SafeTensors(path)
        assert ei.value.status == 1 and "NUL" in str(ei.value)
        return
    stf = abi.SafeTensors(path)
    try:
        assert stf.names() == sorted(tensors)
        for name, (dt, a) in tensors.items():
            ti = stf.info(name)
            assert ti.dtype_name.decode() == dt and tuple(ti.shape[: ti.ndim]) == a.shape
            assert stf.array(name).tobytes() == a.tobytes()
    finally:
        stf.close()


@settings(max_examples=150, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(st.binary(max_size=200), st.integers(0, 300), st.binary(max_size=64))
def test_reader_never_trusts_a_header(tmp_path_factory, header, length, data):
    """Arbitrary header bytes, a declared length that may lie, and trailing data:
    open either succeeds with every entry inside the file or fails with
    YK_ERR_ARG -- never a crash or a read past the mapping."""
    path = tmp_path_factory.mktemp("bad") / "x.safetensors"
    write_raw(path, header, data, length)
    try:
        stf = abi.SafeTensors(path)
    except abi.YKError as e:
        assert e.status == 1
        return
    try:
        size = path.stat().st_size
        for name in stf.names():
            ti = stf.info(name)
            assert ti.nbytes <= size
            stf.array(name)
    finally:
        stf.close()


@settings(max_examples=150, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(st.recursive(st.none() | st.booleans() | st.integers(-2**70, 2**70) | st.floats(allow_nan=False)
                    | st.text(max_size=8),
                    lambda ch: st.lists(ch, max_size=4) | st.dictionaries(st.text(max_size=6), ch, max_size=4),
                    max_leaves=20))
def test_reader_rejects_wrong_structures(tmp_path_factory, value):
    """Well-formed JSON of any shape as the header: accepted only when it really
    describes tensors inside the data block."""
    import json as _json
    path = tmp_path_factory.mktemp("js") / "j.safetensors"
    write_raw(path, _json.dumps(value).encode(), b"\0" * 16)
    try:
        stf = abi.SafeTensors(path)
    except abi.YKError as e:
        assert e.status == 1
        return
    try:
        for name in stf.names():
            ti = stf.info(name)
            assert ti.nbytes <= 16
    finally:
        stf.close()


def test_reader_names_are_utf8(tmp_path):
    """Header text is UTF-8 (JSON): multi-byte names, raw or escaped, come back
    byte-identical; malformed sequences (a stray continuation byte, an overlong
    form, a surrogate, a code point above U+10FFFF, a truncated sequence, 0xFF)
    make the file invalid instead of reaching callers that decode names."""
    arr = np.arange(2, dtype=np.float32)
    p = tmp_path / "u.safetensors"
    names = ["béta", "名前.weight", "x\U0001F600y", "߿ࠀ￿\U0010FFFF"]
    hdr, data = header_and_data({n: ("F32", arr) for n in names})
    for escaped in (False, True):
        write_raw(p, json.dumps(hdr, ensure_ascii=escaped).encode(), data)
        stf = abi.SafeTensors(p)
        try:
            assert stf.names() == sorted(names, key=lambda s: s.encode())
            for n in names:
                assert stf.array(n).tobytes() == arr.tobytes()
        finally:
            stf.close()
    entry = b'": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}'
    for bad in (b"\x80", b"a\xbfb", b"\xc0\xaf", b"\xc1\xbf", b"\xe0\x80\xaf", b"\xed\xa0\x80",
                b"\xf0\x80\x80\xaf", b"\xf4\x90\x80\x80", b"\xf5\x80\x80\x80", b"\xe2\x82", b"\xe2\x82x",
                b"\xff", b"\xfe"):
        write_raw(p, b'{"' + bad + entry, data)
        _expect_invalid(p, "not a JSON object")
