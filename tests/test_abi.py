"""The C-ABI libraries load and export every function include/*.h declares (CPU only;
nothing here launches device work)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from yanaiengine_b200 import abi

ROOT = Path(__file__).resolve().parents[1]


def declared(header: Path) -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return set(re.findall(r"^\s*[A-Za-z_][\w \*]*?\b((?:yk|ykh)_\w+)\s*\(", text, flags=re.M))


def exported(lib: Path) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


@pytest.mark.parametrize("header,lib", [("yk.h", abi.LIB_PATH), ("yk_host.h", abi.HOST_LIB_PATH)])
def test_every_declared_symbol_is_exported(header, lib):
    names = declared(ROOT / "include" / header)
    assert len(names) >= 10
    missing = names - exported(lib)
    assert not missing, f"{lib.name} lacks {sorted(missing)}"
    # and the ctypes binding covers every one of them
    assert names <= set(abi.exported_symbols())


def test_libraries_load_and_bind():
    abi.lib()
    abi.host_lib()
    buf = ctypes.create_string_buffer(64)
    assert abi.lib().yk_last_error(buf, 64) >= 0


def test_config_struct_matches_header():
    text = (ROOT / "include" / "yk.h").read_text()
    body = text[text.index("typedef struct yk_model_config"):text.index("} yk_model_config;")]
    fields = re.findall(r"(?:int32_t|float)\s+(\w+);", body)
    assert fields == [f for f, _ in abi.ModelConfig._fields_]


def test_missing_module_fails_loudly(tmp_path):
    """No CUDA module, no fallback: loading a library that is not built raises."""
    with pytest.raises(RuntimeError, match="not built"):
        abi._load(tmp_path / "libyk.so", {})


def test_null_arguments_are_errors_not_crashes():
    L = abi.lib()
    cfg = abi.ModelConfig()
    assert L.yk_model_get_config(None, ctypes.byref(cfg)) == 1
    assert L.yk_kv_pool_num_blocks(None) == 0
    h = ctypes.c_void_p()
    assert L.yk_safetensors_open(None, ctypes.byref(h)) == 1
    assert L.yk_safetensors_count(None) == 0
    t, l = ctypes.c_int32(), ctypes.c_int32()
    assert L.yk_hf_tensor_id(None, 4, ctypes.byref(t), ctypes.byref(l)) == 1
    assert L.yk_model_load_tensor(None, 0, 0, None, 0, 1, 1, 0) == 1
    H = abi.host_lib()
    assert H.ykh_num_running(None) == 0 and H.ykh_num_waiting(None) == 0
    assert H.ykh_set_window_reclaim(None, 1) == 1
    e = ctypes.c_int32()
    assert H.ykh_step(None, ctypes.byref(e)) == 1


def test_engine_without_a_gpu_reports_an_error():
    """On a machine without a GPU, creating an engine returns an error status (and
    the Python wrapper raises) instead of crashing."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(abi.YKError) as ei:
        abi.Engine(0)
    assert ei.value.status in (1, 3)
