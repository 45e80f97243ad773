"""The C++ CPU backend built with AddressSanitizer + UBSan runs dense, MoE and
hybrid DeltaNet generation and the safetensors reader without a report, and
matches the torch fp32 path token for token."""
import shutil

import pytest


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs the system C++ compiler")
def test_cpu_backend_clean_under_asan_ubsan(tmp_path):
    from mod_b200.utils import sanitize

    out = sanitize.run("address", build_dir=str(tmp_path / "asan"))
    assert "sanitizer run clean" in out
    for name in ("tiny-dense", "tiny-moe", "tiny-next"):
        assert f"{name}: 3/3 sequences token-identical" in out, out[-3000:]
    assert "truncated files rejected" in out
