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
