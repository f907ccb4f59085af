"""bench.py's contract on the CPU: the algorithmic byte counts its roofline divides by, and the
reference arm's JSON line (the reference's own CPU decode, run here on a one-step sample), which
the driver pairs with the GPU arm's line by metric, unit and config."""
import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402
import spmodel  # noqa: E402

REF_SO = os.path.join(ROOT, "oracle", "_ref", "libspref.so")


def test_gemv_bytes_per_token_gemma12b():
    """Codes (half a byte per weight) + f16 block scales + the int8 activations, their block sums
    and the f32 outputs, summed over one token's 48 x (Q|K|V, O, gate+up, down) + the LM head."""
    cfg = spmodel.CONFIGS["gemma12b"]
    shapes = bench.gemv_shapes(cfg)
    assert [s[0] for s in shapes] == ["qkv", "o", "gate_up", "down", "lm_head"]
    assert sum(bench.gemv_bytes(r, c, g) * k for _, r, c, g, k in shapes) == 6626340064
    # one 3840 x 3840 matrix at M = 1: 7372800 code bytes, 921600 scale bytes, 3840 + 480 + 15360
    assert bench.gemv_bytes(3840, 3840, False) == 7372800 + 921600 + 3840 + 480 + 15360


def test_kv_bytes_per_token_gemma12b():
    """40 sliding-window layers read 1024 positions, the 8 global layers the whole context:
    int32 rows (1024 bytes per head) and Spinor rows (5 blocks of 63 bytes)."""
    cfg = spmodel.CONFIGS["gemma12b"]
    assert bench.kv_bytes_per_token(cfg, 2052, 1024) == (40 * 1024 + 8 * 2052) * 8 * 2 * 1024
    assert bench.kv_bytes_per_token(cfg, 512, 315) == 48 * 512 * 8 * 2 * 315
    q = spmodel.CONFIGS["qwen8b"]   # no sliding window: every layer reads the whole context
    assert bench.kv_bytes_per_token(q, 4096, 512) == 36 * 4096 * 8 * 2 * 512


def test_reference_arm_other_ranks_print_nothing():
    env = dict(os.environ, RANK="1", LOCAL_RANK="1", WORLD_SIZE="2")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="oracle/_ref/libspref.so not built")
def test_reference_arm_line():
    """One timed step: the line carries the GPU arm's metric, unit and workload, a measured
    ms_per_step, the cpu_baseline object and an e2e object with no host-device bytes."""
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "tokens/s"
    assert line["higher_is_better"] is True and line["steps"] == 1 and line["warmup"] == 1
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert "configs[2]" in line["config"]["workload"]
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] == "reference" and cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    # the unscaled configs[0] figures of the reference and of the checker, one core each
    for k in ("reference", "xref"):
        c1 = line["config1_unscaled"][k]
        assert c1["decode_tokens_per_s"] > 0 and c1["cores"] == 1 and c1["scaled"] is False


def _gpu_usable():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_gpu_usable(), reason="checks the behaviour without a GPU")
def test_gpu_arm_fails_loudly_without_a_gpu():
    """No CPU fallback: without a GPU the device arm exits nonzero and prints no bench line."""
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--steps", "1", "--warmup", "1"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode != 0
    assert r.stdout.strip() == ""
