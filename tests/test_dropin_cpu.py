"""The drop-in patch (oracle/dropin_patch.py) adds the INTEGRATION.md seams
and changes nothing else in the reference's tinylm.c.  CPU only; needs the
reference sources (build machine)."""
import os
import re
import subprocess

import pytest

import oracle

pytestmark = pytest.mark.skipif(not os.path.exists(oracle.REF_SRC), reason="reference sources not present")
HERE = os.path.dirname(os.path.abspath(__file__))


def patched(tmp_path):
    out = tmp_path / "tinylm.c"
    subprocess.run(["python", os.path.join(oracle.HERE, "dropin_patch.py"), oracle.REF_SRC, str(out)], check=True)
    return open(oracle.REF_SRC).read(), out.read_text()


def test_patch_only_inserts_the_seams(tmp_path):
    src, dst = patched(tmp_path)
    blocks = re.findall(r"\n#ifdef USE_CUDA\n.*?\n#endif\n", dst, flags=re.S)
    assert len(blocks) == 6                   # header block + mm, mm_bt, mm_atb, adamw, global_gradnorm
    stripped = dst
    for b in blocks:
        stripped = stripped.replace(b, "\n", 1)
    assert re.sub(r"\n+", "\n", stripped) == re.sub(r"\n+", "\n", src)
    calls = "".join(blocks)
    for fn in ("tl_matmul(Y, X, W, M, K, N)", "tl_matmul_bt(dX, dY, W, M, K, N)", "tl_matmul_at(dW, X, dY, M, K, N)",
               "tl_adamw_step(P, G, M, Vv, n, lr, b1, b2, wd, t, gscale)", "tl_grad_norm(G, n, &nrm)",
               "tl_set_host_buffers(1)"):
        assert fn in calls, fn


def test_patched_copy_without_use_cuda_is_the_reference(tmp_path):
    """-DUSE_CUDA off: the preprocessed copy equals the preprocessed reference."""
    src, dst = patched(tmp_path)
    flags = ["-E", "-P", "-w", "-I" + os.path.join(oracle.HERE, "shim"), "-D__declspec(x)=", "-D__stdcall="]
    a = subprocess.run(["gcc", *flags, oracle.REF_SRC], capture_output=True, text=True, check=True).stdout
    b = subprocess.run(["gcc", *flags, str(tmp_path / "tinylm.c")], capture_output=True, text=True, check=True).stdout
    assert a.split() == b.split()
