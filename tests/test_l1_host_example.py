"""The host-side registration (tests/l1_host_example.c, the C that INTEGRATION.md shows a
maintainer adding) compiled against the reference's frozen L1 headers and linked with the
reference's own library and libspb200_l1.so. On a machine without a usable GPU every device
call must come back as a status: the reference session's prefill as SP_EBADSTATE (-4) carrying
the backend's detail (sp_session.c:198-206), the section-6b open as nonzero, and no crash."""
import os
import subprocess

import pytest

import spmodel
from conftest import ROOT

PKG = os.path.join(ROOT, "shannon-prime-system_b200")
L1_SO = os.path.join(PKG, "libspb200_l1.so")
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libspref.so")
REF_INCLUDE = os.environ.get("SPB_REF_INCLUDE", os.path.join(os.path.dirname(ROOT), "reference", "include"))


def _gpu_usable():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="module")
def example(tmp_path_factory):
    for p in (L1_SO, REF_SO, os.path.join(REF_INCLUDE, "sp", "sp_l1.h")):
        if not os.path.exists(p):
            pytest.skip(f"{p} absent")
    d = tmp_path_factory.mktemp("l1ex")
    exe = str(d / "l1_host_example")
    cmd = ["gcc", "-std=c11", "-O1", "-Wall", "-Werror", "-I", REF_INCLUDE, "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "l1_host_example.c"), "-o", exe, REF_SO, L1_SO,
           f"-Wl,-rpath,{os.path.dirname(REF_SO)}:{PKG}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    cfg = spmodel.CONFIGS["micro_gemma"]
    mp, tp = str(d / "m.sp-model"), str(d / "m.sp-tokenizer")
    spmodel.write_sp_model(mp, tp, cfg, spmodel.gen_model(cfg, seed=0))
    return exe, mp, tp, d


def test_example_compiles_against_the_frozen_headers(example):
    exe, _, _, _ = example
    assert os.access(exe, os.X_OK)


@pytest.mark.skipif(_gpu_usable(), reason="checks the no-GPU statuses")
def test_example_without_gpu_reports_statuses(example):
    exe, mp, tp, d = example
    out = str(d / "logits.f32")
    r = subprocess.run([exe, mp, tp, "9", out], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, (r.stdout, r.stderr)
    lines = dict(l.split(" ", 1) for l in r.stdout.strip().splitlines())
    assert lines["register6"] == "0"
    rc, detail = lines["prefill6"].split(" ", 1)
    assert int(rc) == -4 and "spb200" in detail      # SP_EBADSTATE with the backend's detail
    assert not lines["open6b"].startswith("0")
    assert lines["done"] == "1"
    assert not os.path.exists(out)                   # nothing written when a call failed
