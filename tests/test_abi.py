"""The C-ABI library loads on CPU and exports every symbol the public header declares."""
import re
import subprocess
from pathlib import Path

import bonsai_b200 as bb

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    text = (ROOT / "include" / "bonsai_cuda.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bonsai_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    if not bb.LIB_PATH.exists():
        subprocess.run(["make", "-C", str(ROOT / "bonsai.cpp_b200")], check=True,
                       capture_output=True)
    L = bb.lib()
    names = declared_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, f"declared but not exported: {missing}"
    assert set(names) == set(bb.SIGNATURES), "ctypes signature table out of sync with the header"


def test_no_gpu_error_paths():
    """Argument validation runs before any device work: a bad call returns
    an error code and a message instead of aborting (the reference aborts,
    src/b1_0_kernel.h:195-198)."""
    L = bb.lib()
    import ctypes
    h = ctypes.c_void_p()
    rc = L.bonsai_b1_upload(None, 32, 64, -1, ctypes.byref(h))
    assert rc == -1 and b"null" in L.bonsai_last_error()
    buf = (ctypes.c_uint8 * (32 * 3 * 6))()
    rc = L.bonsai_b1_upload(buf, 32, 96 + 1, -1, ctypes.byref(h))
    assert rc == -1 and b"multiple of 32" in L.bonsai_last_error()
    assert L.bonsai_b1_gemm(None, 64, 4, None, 0, None, 32, None, None) == -1
    assert L.bonsai_joint_attention(None, None, None, 24, 128, 64, 0.1, None, 3072, None) == -2
    assert L.bonsai_dit_set_weight(None, b"img_in.w", None, 0) == -1
    assert L.bonsai_dit_load_safetensors(None, b"/nonexistent.safetensors") == -1
    assert L.bonsai_dit_sample(None, None, None, None, 4, None, None) == -1
    assert L.bonsai_count_nonfinite(None, 5, None, None) == -1
    assert b"count_nonfinite" in L.bonsai_last_error()
