"""Generate the golden vectors under tests/golden/ by running the reference's own
compiled code (oracle/_ref/libspref.so, built from the reference sources by
`make -C oracle ref`). Re-run: python tests/golden/make_golden.py [spinor | fidelity]

Every vector is (seeded input, reference output). The CPU test-suite checks the XREF
restatement against them, so XREF stays pinned where the reference tree is absent.
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "shannon-prime-system_b200"))
import spmodel  # noqa: E402
import xref  # noqa: E402


def main():
    C.CDLL(xref.SPREF_SO, mode=C.RTLD_GLOBAL)
    R = xref.RefLib()
    L = R.lib
    rng = np.random.default_rng(20261201)
    out = {}
    # ---- islands (exact_islands.c:60-124), the T_EXACT_ISLANDS sizes and a scale sweep
    cases = [(3840, 1.0), (3840, 0.01), (4096, 3.0), (512, 40.0), (256, 0.3), (64, 1.0), (128, 7.0),
             (1, 2.0), (37, 0.5), (15360, 1.0)]
    for i, (n, sc) in enumerate(cases):
        x = (rng.standard_normal(n) * sc).astype(np.float32)
        w = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        y = np.empty(n, np.float32)
        L.sp_rmsnorm_exact(x.ctypes.data, w.ctypes.data, n, y.ctypes.data)
        out[f"rms{i}_x"], out[f"rms{i}_w"], out[f"rms{i}_y"] = x, w, y
    for i, (m, sc) in enumerate([(256, 3.0), (1024, 10.0), (1, 1.0), (8192, 5.0), (33, 0.01)]):
        z = (rng.standard_normal(m) * sc).astype(np.float32)
        p = np.empty(m, np.float64)
        L.sp_softmax_exact(z.ctypes.data, m, p.ctypes.data)
        out[f"sm{i}_z"], out[f"sm{i}_p"] = z, p
    for i, (n, sc) in enumerate([(512, 1.0), (4096, 4.0), (2048, 0.05), (1000, 30.0)]):
        x = (rng.standard_normal(n) * sc).astype(np.float32)
        y = np.empty(n, np.float32)
        L.sp_gelu_exact(x.ctypes.data, n, y.ctypes.data)
        out[f"gelu{i}_x"], out[f"gelu{i}_y"] = x, y
    # ---- codec: every f16 (weight_dtype.c:9-28) and the quantizer (frobenius_lift.c:27-35)
    h = np.arange(65536, dtype=np.uint16)
    f = np.array([L.sp_f16_to_f32(int(v)) for v in h], np.float32)
    out["f16_bits"], out["f16_f32"] = h, f
    v = (rng.standard_normal(20000) * 3).astype(np.float32)
    s = np.float32(np.abs(v).max())
    v[:6] = [s, -s, 0.0, s / 254, -s / 254, s * 0.999]
    q = np.array([L.sp_frob_quant1(float(a), float(s)) for a in v], np.int8)
    out["q1_v"], out["q1_s"], out["q1_q"] = v, np.array([s], np.float32), q
    # ---- Q4 unpack (frobenius_lift.c:102-107)
    nib = rng.integers(0, 256, 64, dtype=np.uint8)
    codes = np.empty(128, np.int8)
    L.sp_frob_q4_unpack.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
    L.sp_frob_q4_unpack(nib.ctypes.data, 128, codes.ctypes.data)
    out["unpack_nib"], out["unpack_codes"] = nib, codes
    # ---- hashes of the .sp-model format (sp_hash.c)
    names = [b"", b"token_embd.weight", b"blk.0.attn_q.weight.bscale", bytes(range(97))]
    out["xxh64"] = np.array([L.sp_xxh64(n, len(n), 0) for n in names], np.uint64)
    out["crc32"] = np.array([L.sp_crc32(n, len(n)) for n in names], np.uint32)
    # ---- reference float forward on the micro models (fidelity, not a byte gate)
    for name in ("micro_gemma", "micro_qwen"):
        cfg = spmodel.CONFIGS[name]
        T = spmodel.gen_model(cfg, seed=0)
        mp, tp = f"/tmp/golden_{name}.sp-model", f"/tmp/golden_{name}.sp-tokenizer"
        spmodel.write_sp_model(mp, tp, cfg, T)
        m = R.load(mp, tp)
        sess = R.session(m, cfg.max_context)
        toks = spmodel.gen_tokens(11, 20, cfg.n_vocab)
        rc, lg = R.prefill(sess, toks, cfg.n_vocab)
        assert rc == 0, R.err()
        out[f"fwd_{name}_tokens"], out[f"fwd_{name}_logits"] = toks, lg
    np.savez_compressed(os.path.join(HERE, "reference_vectors.npz"), **out)
    print("wrote", len(out), "arrays")


SPINOR_LENS = [1, 7, 43, 54, 55, 56, 64, 110, 111, 128, 200, 256]


def spinor_inputs(rng):
    """Seeded head rows for the Spinor KV codec: float rows at several scales (zeros, exact
    rounding ties and saturation included), and K rows on the 2^16 score grid."""
    rows = []
    for k in SPINOR_LENS:
        for sc in (1e-3, 1.0, 300.0):
            rows.append((rng.standard_normal(k) * sc).astype(np.float32))
        v = rng.integers(-254, 255, k).astype(np.float32) / 2.0   # halves: rounding ties
        v[0] = 127.0
        rows.append(v)
        z = np.zeros(k, np.float32)
        rows.append(z)
        if k > 3:
            z2 = (rng.standard_normal(k) * 5).astype(np.float32)
            z2[::3] = 0.0
            z2[1] = -0.0
            rows.append(z2)
    grids = [rng.integers(-(1 << 24) + 1, 1 << 24, k).astype(np.int32) for k in (64, 128, 256)]
    grids += [(rng.standard_normal(256) * 65536 * 3).astype(np.int32)]
    return rows, grids


def spinor():
    """Spinor blocks from the reference's own codec (core/vht2/spinor_block.c, vht2.c,
    mobius_reorder.c): encode_vec and decode_vec of every seeded row."""
    C.CDLL(xref.SPREF_SO, mode=C.RTLD_GLOBAL)
    L = C.CDLL(xref.SPREF_SO)
    L.sp_spinor_encode_vec.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
    L.sp_spinor_decode_vec.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
    rows, grids = spinor_inputs(np.random.default_rng(20261202))
    out = {}
    for i, v in enumerate(rows + [g.astype(np.float32) * np.float32(1.0 / 65536) for g in grids]):
        nb = 1 if v.size <= 55 else (v.size + 54) // 55
        blk = np.zeros(nb * 63, np.uint8)
        L.sp_spinor_encode_vec(v.ctypes.data, v.size, blk.ctypes.data)
        dec = np.zeros(v.size, np.float32)
        rc = L.sp_spinor_decode_vec(blk.ctypes.data, v.size, dec.ctypes.data)
        assert rc == 0
        out[f"sp{i}_v"], out[f"sp{i}_blocks"], out[f"sp{i}_dec"] = v, blk, dec
    np.savez_compressed(os.path.join(HERE, "spinor_vectors.npz"), **out)
    print("wrote", len(out), "arrays")


# (case, base config, overrides, prompt tokens): the width the bench runs at, cut to a few layers and
# a 4096-token vocabulary so the reference float forward finishes in seconds; gemma12b keeps six
# layers so its global layer (L % 6 == 5, sp_session.c:396) is among them
FIDELITY_CASES = [
    ("tiny", "tiny", {}, 32),
    ("gemma12b_w6", "gemma12b", {"n_layers": 6, "n_vocab": 4096, "max_context": 64}, 8),
    ("qwen8b_w4", "qwen8b", {"n_layers": 4, "n_vocab": 4096, "max_context": 64}, 8),
]


def fidelity():
    """The reference float forward (sp_prefill_chunk with no backend) at BASELINE configs[0] and
    at the 12B and 8B widths: the last prompt row's logits, for XREF's fidelity test."""
    import dataclasses
    C.CDLL(xref.SPREF_SO, mode=C.RTLD_GLOBAL)
    R = xref.RefLib()
    out = {}
    for name, base, kw, n in FIDELITY_CASES:
        cfg = dataclasses.replace(spmodel.CONFIGS[base], **kw)
        T = spmodel.gen_model(cfg, seed=0)
        mp, tp = f"/tmp/fidelity_{name}.sp-model", f"/tmp/fidelity_{name}.sp-tokenizer"
        spmodel.write_sp_model(mp, tp, cfg, T)
        m = R.load(mp, tp)
        sess = R.session(m, cfg.max_context)
        toks = spmodel.gen_tokens(12, n, cfg.n_vocab)
        rc, lg = R.prefill(sess, toks, cfg.n_vocab)
        assert rc == 0, R.err()
        out[f"{name}_tokens"], out[f"{name}_logits"] = toks, lg
        R.lib.sp_session_destroy(sess)
        R.lib.sp_model_unload(m)
        os.remove(mp)
        os.remove(tp)
    np.savez_compressed(os.path.join(HERE, "fidelity_vectors.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    if sys.argv[1:] == ["spinor"]:
        spinor()
    elif sys.argv[1:] == ["fidelity"]:
        fidelity()
    else:
        main()
