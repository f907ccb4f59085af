"""The drop-in boundary without a GPU: every symbol include/*.h declares is exported by
the built libraries, the .sp-model writer round-trips through the reference loader, and
the reference session runs the written OK_Q4B models."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import spb200
import spmodel
from conftest import ROOT


def declared(header):
    txt = open(os.path.join(ROOT, "include", header)).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(spb_\w+)\s*\(", txt)))


def exported(so):
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True).stdout
    return {l.split()[-1] for l in out.splitlines() if " T " in l}


def test_core_library_exports_every_declared_symbol():
    names = declared("spb200.h")
    assert set(names) == set(spb200.CORE_SYMBOLS)
    missing = [n for n in names if n not in exported(spb200.CORE_SO)]
    assert not missing, missing
    spb200.load()   # loads without a GPU


def test_l1_library_exports_every_declared_symbol():
    if not os.path.exists(spb200.L1_SO):
        pytest.skip("libspb200_l1.so not built (reference headers absent at build time)")
    names = declared("spb200_l1.h")
    assert set(names) == set(spb200.L1_SYMBOLS)
    missing = [n for n in names if n not in exported(spb200.L1_SO)]
    assert not missing, missing


def test_no_device_is_a_clean_error(spb):
    if spb.spb_device_count() > 0:
        pytest.skip("a GPU is visible")
    h = C.c_void_p()
    cfg = spb200.config_struct(spmodel.CONFIGS["micro_qwen"])
    rc = spb.spb_model_synthetic(C.byref(cfg), 0, 0, C.byref(h))
    assert rc in (spb200.SPB_ECUDA, spb200.SPB_EOOM) and spb.spb_last_error()


def test_bad_shapes_rejected_before_any_device_call(spb):
    import dataclasses
    bad = dataclasses.replace(spmodel.CONFIGS["micro_qwen"], head_dim=48)
    h = C.c_void_p()
    rc = spb.spb_model_synthetic(C.byref(spb200.config_struct(bad)), 0, 0, C.byref(h))
    assert rc == spb200.SPB_EUNSUPPORTED
    assert b"head_dim" in spb.spb_last_error()
    assert spb.spb_gemv_q4b(None, None, 1, 33, None, 1, None, None) == spb200.SPB_EBADARG


def test_generator_is_deterministic_and_uniform():
    a = spmodel.gen_codes(0, 10, 64, 512)
    b = spmodel.gen_codes(0, 10, 64, 512)
    assert np.array_equal(a, b)
    nib = np.concatenate([a.ravel() & 15, a.ravel() >> 4])
    counts = np.bincount(nib, minlength=16)
    assert counts.min() > 0.9 * counts.mean()          # all 16 code values, incl. -8
    s = spmodel.gen_bscale(0, 11, 64, 512).astype(np.uint32)
    e = (s >> 10) & 31
    assert np.all(e == spmodel.scale_exponent(512) + 15)
    neg = (s >> 15) & 1                                  # random signs: no common-mode row offset
    assert 0.45 < neg.mean() < 0.55
    w = spmodel.gen_norm(0, 12, 1000)
    assert w.min() >= 0.9 and w.max() < 1.1


def test_sp_model_roundtrip_through_reference_loader(reflib, tmp_path):
    cfg = spmodel.CONFIGS["micro_qwen"]
    T = spmodel.gen_model(cfg, seed=2)
    mp, tp = str(tmp_path / "m.sp-model"), str(tmp_path / "m.sp-tokenizer")
    spmodel.write_sp_model(mp, tp, cfg, T)
    L = reflib.lib
    m = reflib.load(mp, tp)
    L.sp_model_find_tensor.argtypes = [C.c_void_p, C.c_char_p]
    L.sp_model_find_tensor.restype = C.c_void_p
    L.sp_model_tensor_data.argtypes = [C.c_void_p, C.c_void_p]
    L.sp_model_tensor_data.restype = C.c_void_p
    for name in ["blk.1.ffn_down.weight", "token_embd.weight", "output_norm.weight"]:
        e = L.sp_model_find_tensor(m, name.encode())
        assert e
        p = L.sp_model_tensor_data(m, e)
        t = T[name]
        arr = t.codes if isinstance(t, spmodel.Q4B) else t
        got = np.ctypeslib.as_array((C.c_uint8 * arr.nbytes).from_address(p))
        assert np.array_equal(got, arr.view(np.uint8).ravel())
    e = L.sp_model_find_tensor(m, b"blk.1.ffn_down.weight.bscale")
    p = L.sp_model_tensor_data(m, e)
    got = np.ctypeslib.as_array((C.c_uint16 * T["blk.1.ffn_down.weight"].bscale.size).from_address(p))
    assert np.array_equal(got, T["blk.1.ffn_down.weight"].bscale.ravel())
    L.sp_model_unload(m)


def test_corrupted_header_rejected(reflib, tmp_path):
    cfg = spmodel.CONFIGS["micro_qwen"]
    T = spmodel.gen_model(cfg, seed=2)
    mp, tp = str(tmp_path / "m.sp-model"), str(tmp_path / "m.sp-tokenizer")
    spmodel.write_sp_model(mp, tp, cfg, T)
    raw = bytearray(open(mp, "rb").read())
    raw[30] ^= 0xFF          # inside arch_struct -> CRC mismatch
    open(mp, "wb").write(raw)
    with pytest.raises(RuntimeError, match="CRC"):
        reflib.load(mp, tp)
