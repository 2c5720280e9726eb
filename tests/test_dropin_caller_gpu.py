"""A compiled C++ caller of the C ABI (oracle/dropin_caller.cpp, built by
`make -C oracle` from the reference's own headers through the ggml shim):
the reference's node factories b1_linear() / rope_2d_fwd()
(src/b1_0_kernel.h:290-300, :363-371) build custom nodes, a miniature CUDA
backend dispatches them by the magic in their user data to
bonsai_b1_linear_f32 / bonsai_rope_2d_f32, and the results are compared with
the same nodes run through their own CPU callbacks (the reference's kernels).
"""
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

BIN = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "dropin_caller"


def test_compiled_caller_dispatches_reference_nodes(gpu):
    assert BIN.exists(), (f"{BIN} is missing: build it with `make -C oracle` where the reference "
                          "checkout is readable (BONSAI_REF_DIR)")
    r = subprocess.run([str(BIN)], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL OK" in r.stdout
    assert r.stdout.count(" ok") == 5, r.stdout
