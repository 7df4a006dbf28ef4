"""bench.py's output contract, checked on the CPU through its reference arm:
stdout carries exactly one JSON line (whatever libraries print goes to
stderr), with the keys the reference arm's line must have."""
import json
import os
import subprocess
import sys

import pytest

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not oracle.has_ref(), reason="reference leg not built")
def test_reference_arm_prints_one_json_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "gemm",
                        "--shape", "64,64,64", "--steps", "1", "--warmup", "3"],
                       capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.splitlines()
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and isinstance(d["value"], (int, float)) and d["value"] >= 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


@pytest.mark.skipif(not oracle.has_ref(), reason="reference leg not built")
def test_library_output_on_fd1_goes_to_stderr():
    """What a C library writes to file descriptor 1 during the run (NCCL's
    version banner) must not reach bench.py's stdout."""
    code = ("import os, sys\n"
            "sys.argv = ['bench.py', '--impl', 'reference', '--workload', 'gemm', '--shape', '64,64,64', "
            "'--steps', '1', '--warmup', '3']\n"
            f"sys.path.insert(0, {ROOT!r})\n"
            "import bench\n"
            "def noisy():\n"
            "    os.write(1, b'BANNER from a library\\n')\n"
            "    return bench.main()\n"
            "sys.exit(bench.run_as_script(noisy))\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "BANNER" not in r.stdout and "BANNER" in r.stderr
    assert len(r.stdout.splitlines()) == 1


def _bench():
    sys.path.insert(0, ROOT)
    import bench
    return bench


def test_gemm_ceiling_follows_the_split():
    """The roofline denominators: 3xTF32 = bf16 / 6 (three tf32 passes at half
    the bf16 rate); the hybrid split = bf16 / 4 (one tf32 pass, one bf16 pass
    over twice the K), which the training workloads use under the automatic
    choice; the fp16 split = bf16 / 3."""
    b = _bench()
    assert b.gemm_ceiling(0)[0] == 6.0
    assert b.gemm_ceiling(3)[0] == 6.0
    assert b.gemm_ceiling(3, training=True)[0] == 6.0
    assert b.gemm_ceiling(0, training=True)[0] == 4.0
    assert b.gemm_ceiling(5)[0] == 4.0
    assert b.gemm_ceiling(4)[0] == 3.0
    assert "hybrid" in b.gemm_ceiling(0, training=True)[1]


def test_gemm_flops_per_token_config5():
    """6 x the GEMM-held parameters per token: 1.1325 GFLOP for the scaled
    tiny Llama (V 8192, D 1024, 16 layers, 16 / 4 heads, F 2816, no MTP), and
    the m1 preset's 8.99 MFLOP with two MTP heads."""
    b = _bench()
    assert b.gemm_flops_per_token((8192, 1024, 16, 16, 4, 2816, 256, 0)) == 1132462080
    m1 = b.gemm_flops_per_token((2048, 128, 4, 4, 1, 336, 256, 2))
    assert abs(m1 / 1e6 - 8.99) < 0.01
