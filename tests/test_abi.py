"""The C-ABI library loads and exports every symbol include/zkml_b200.h declares."""
import re
import subprocess
from pathlib import Path

import zkml_b200 as Z

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    hdr = (ROOT / "include" / "zkml_b200.h").read_text()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    return sorted(set(re.findall(r"\b(zkml_[a-z0-9_]+)\s*\(", hdr)))


def test_header_and_binding_agree():
    assert declared_functions() == sorted(Z.exported_symbols())


def test_library_exports_every_declared_symbol():
    L = Z.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(Z.library_path())], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (zkml_\w+)", out))
    assert set(declared_functions()) <= exported


def test_abi_version():
    assert Z.lib().zkml_abi_version() == 1


def test_ctx_create_without_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        return
    try:
        Z.Context(0)
    except Z.ZkmlError as e:
        assert e.status in (3, 6)
    else:
        raise AssertionError("context creation must fail without a GPU")
