"""ctypes bindings for the checkers under oracle/ (test infrastructure only).

* `Xref`      -- the exact-integer CPU forward (oracle/_ref/libxref.so, built from
                 oracle/*.c by `make -C oracle`).
* `RefLib`    -- the reference's own L1 math core (oracle/_ref/libspref.so, compiled
                 from the reference sources by the same Makefile when the reference
                 tree is present): sp_model_load / sp_session_* / sp_prefill_chunk /
                 sp_decode_step, the float forward the byte-exact path is a
                 fidelity-replacement of, plus its exact islands and hashes.

Nothing in the product library imports this module.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
XREF_SO = os.path.join(REF_DIR, "libxref.so")
SPREF_SO = os.path.join(REF_DIR, "libspref.so")

XREF_OK, XREF_EBADARG, XREF_ERANGE = 0, -3, -50

_fp = C.POINTER(C.c_float)
_ip = C.POINTER(C.c_int32)


class XQ4B(C.Structure):
    _fields_ = [("codes", C.c_void_p), ("bscale", C.c_void_p), ("rows", C.c_int32), ("cols", C.c_int32)]


class XLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("attn_norm", "q_norm", "k_norm", "post_attn_norm",
                                          "ffn_norm", "post_ffw_norm")] + \
               [(n, XQ4B) for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd")]


class XConfig(C.Structure):
    _fields_ = [("arch", C.c_int32), ("n_layers", C.c_int32), ("n_embd", C.c_int32),
                ("n_ff", C.c_int32), ("n_head", C.c_int32), ("n_head_kv", C.c_int32),
                ("head_dim", C.c_int32), ("n_vocab", C.c_int32), ("sliding_window", C.c_int32),
                ("rope_base", C.c_float), ("rope_base_local", C.c_float),
                ("swa_period", C.c_int32), ("has_qk_norm", C.c_int32)]


class XModel(C.Structure):
    _fields_ = [("cfg", XConfig), ("layers", C.c_void_p), ("token_embd", XQ4B),
                ("output", XQ4B), ("output_norm", C.c_void_p)]


_LAYER_MAP = [("attn_norm", "attn_norm"), ("q_norm", "attn_q_norm"), ("k_norm", "attn_k_norm"),
              ("post_attn_norm", "post_attention_norm"), ("ffn_norm", "ffn_norm"),
              ("post_ffw_norm", "post_ffw_norm")]
_MAT_MAP = [("wq", "attn_q"), ("wk", "attn_k"), ("wv", "attn_v"), ("wo", "attn_output"),
            ("wg", "ffn_gate"), ("wu", "ffn_up"), ("wd", "ffn_down")]


def _ptr(a):
    return None if a is None else a.ctypes.data


def _q4b(t, struct_type):
    return struct_type(_ptr(t.codes), _ptr(t.bscale), t.rows, t.cols)


def build_desc(cfg, T, struct_types=(XQ4B, XLayer, XConfig, XModel)):
    """Descriptor over the numpy tensors of gen_model(); keeps the arrays alive."""
    Q, Ly, Cf, Md = struct_types
    layers = (Ly * cfg.n_layers)()
    for L in range(cfg.n_layers):
        ly = layers[L]
        for f, nm in _LAYER_MAP:
            t = T.get(f"blk.{L}.{nm}.weight")
            setattr(ly, f, _ptr(t))
        for f, nm in _MAT_MAP:
            setattr(ly, f, _q4b(T[f"blk.{L}.{nm}.weight"], Q))
    out = T.get("output.weight", T["token_embd.weight"])
    cf = Cf(cfg.arch, cfg.n_layers, cfg.n_embd, cfg.n_ff, cfg.n_head, cfg.n_head_kv,
            cfg.head_dim, cfg.n_vocab, cfg.sliding_window, cfg.rope_base,
            cfg.rope_base_local, cfg.swa_period, cfg.has_qk_norm)
    m = Md(cf, C.addressof(layers), _q4b(T["token_embd.weight"], Q), _q4b(out, Q),
           _ptr(T["output_norm.weight"]))
    m._keep = (layers, T)
    return m


class Xref:
    def __init__(self, path=XREF_SO):
        self.lib = L = C.CDLL(path)
        L.xref_session_create.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_void_p)]
        L.xref_session_destroy.argtypes = [C.c_void_p]
        L.xref_decode_step.argtypes = [C.c_void_p, C.c_int32, C.c_void_p]
        L.xref_prefill.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.xref_rewind.argtypes = [C.c_void_p, C.c_int]
        L.xref_position.argtypes = [C.c_void_p]
        L.xref_clone.argtypes = [C.c_void_p, C.POINTER(C.c_void_p)]
        L.xref_kv_read.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
        L.xref_matvec.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.xref_matvec_q.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.xref_quant_vec.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        L.xref_rmsnorm_exact.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.xref_softmax_exact.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.xref_gelu_exact.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.xref_silu_exact.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.xref_rope_freq_table.argtypes = [C.c_float, C.c_int, C.c_void_p]
        L.xref_rope_cordic.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_void_p, C.c_void_p]
        L.xref_cordic_atan_table.argtypes = [C.c_void_p]
        L.xref_cordic_gain_q62.restype = C.c_uint64
        L.xref_attn_head.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                     C.c_int, C.c_int, C.c_float, C.c_void_p]
        L.xref_session_create_ex.argtypes = [C.c_void_p, C.c_int, C.c_uint, C.POINTER(C.c_void_p)]
        L.xref_kv_bytes.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
        L.xref_crc8.argtypes = [C.c_void_p, C.c_int]
        L.xref_crc8.restype = C.c_uint8
        L.xref_spinor_encode_vec.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.xref_spinor_decode_vec.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.xref_spinor_kv_row.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]

    # ---- Spinor KV blocks
    @staticmethod
    def spinor_blocks_for(k):
        return 1 if k <= 55 else (k + 54) // 55

    def spinor_encode(self, v):
        v = np.ascontiguousarray(v, np.float32)
        o = np.zeros(self.spinor_blocks_for(v.size) * 63, np.uint8)
        self.lib.xref_spinor_encode_vec(v.ctypes.data, v.size, o.ctypes.data)
        return o

    def spinor_decode(self, blocks, k):
        blocks = np.ascontiguousarray(blocks, np.uint8)
        o = np.zeros(k, np.float32)
        rc = self.lib.xref_spinor_decode_vec(blocks.ctypes.data, k, o.ctypes.data)
        return o, rc

    def spinor_kv_row(self, hd, kg=None, vf=None):
        """(blocks, grid, rc) of one head row: a K row on the 2^16 grid, or a V row of floats."""
        blocks = np.zeros(self.spinor_blocks_for(hd) * 63, np.uint8)
        grid = np.zeros(hd, np.int32)
        kp = np.ascontiguousarray(kg, np.int32) if kg is not None else None
        vp = np.ascontiguousarray(vf, np.float32) if vf is not None else None
        rc = self.lib.xref_spinor_kv_row(kp.ctypes.data if kp is not None else None,
                                         vp.ctypes.data if vp is not None else None, hd,
                                         blocks.ctypes.data, grid.ctypes.data)
        return blocks, grid, rc

    # ---- elementwise helpers on numpy arrays
    def rmsnorm(self, x, w):
        x = np.ascontiguousarray(x, np.float32); w = np.ascontiguousarray(w, np.float32)
        o = np.empty_like(x); self.lib.xref_rmsnorm_exact(x.ctypes.data, w.ctypes.data, x.size, o.ctypes.data)
        return o

    def gelu(self, x):
        x = np.ascontiguousarray(x, np.float32); o = np.empty_like(x)
        self.lib.xref_gelu_exact(x.ctypes.data, x.size, o.ctypes.data); return o

    def silu(self, x):
        x = np.ascontiguousarray(x, np.float32); o = np.empty_like(x)
        self.lib.xref_silu_exact(x.ctypes.data, x.size, o.ctypes.data); return o

    def softmax(self, z):
        z = np.ascontiguousarray(z, np.float32); p = np.empty(z.size, np.float64)
        self.lib.xref_softmax_exact(z.ctypes.data, z.size, p.ctypes.data); return p

    def quant(self, u):
        u = np.ascontiguousarray(u, np.float32); q = np.empty(u.size, np.int8); s = np.zeros(1, np.float32)
        self.lib.xref_quant_vec(u.ctypes.data, u.size, q.ctypes.data, s.ctypes.data); return q, float(s[0])

    def matvec(self, t, X):
        X = np.ascontiguousarray(X, np.float32).reshape(-1, t.cols)
        Y = np.empty((X.shape[0], t.rows), np.float32)
        d = _q4b(t, XQ4B)
        rc = self.lib.xref_matvec(C.byref(d), X.ctypes.data, X.shape[0], Y.ctypes.data)
        if rc:
            raise RuntimeError(f"xref_matvec rc={rc}")
        return Y

    def q4b_check(self, t):
        """0 when every row keeps the exact int64 accumulation bound, else -1 (xref_q4b_check)."""
        return int(self.lib.xref_q4b_check(C.byref(_q4b(t, XQ4B))))

    def matvec_q(self, t, q, s):
        q = np.ascontiguousarray(q, np.int8).reshape(-1, t.cols); s = np.ascontiguousarray(s, np.float32)
        Y = np.empty((q.shape[0], t.rows), np.float32)
        self.lib.xref_matvec_q(C.byref(_q4b(t, XQ4B)), q.ctypes.data, s.ctypes.data, q.shape[0], Y.ctypes.data)
        return Y

    def rope_table(self, base, d):
        W = np.zeros(d // 2, np.uint64)
        rc = self.lib.xref_rope_freq_table(base, d, W.ctypes.data)
        if rc:
            raise RuntimeError(f"rope table rc={rc}")
        return W

    def rope(self, v, p, W):
        v = np.ascontiguousarray(v, np.float32); o = np.zeros(v.size, np.int32)
        rc = self.lib.xref_rope_cordic(v.ctypes.data, v.size, p, W.ctypes.data, o.ctypes.data)
        return o, rc

    # ---- sessions
    def session(self, desc, max_ctx, spinor=False):
        return XrefSession(self, desc, max_ctx, flags=1 if spinor else 0)


class XrefSession:
    def __init__(self, xr, desc, max_ctx, handle=None, flags=0):
        self.xr, self.desc, self.max_ctx, self.flags = xr, desc, max_ctx, flags
        self.V = desc.cfg.n_vocab
        if handle is None:
            h = C.c_void_p()
            rc = xr.lib.xref_session_create_ex(C.byref(desc), max_ctx, flags, C.byref(h))
            if rc:
                raise RuntimeError(f"xref_session_create rc={rc}")
            handle = h
        self.h = handle

    def close(self):
        if self.h:
            self.xr.lib.xref_session_destroy(self.h)
            self.h = None

    __del__ = close

    def step(self, tok):
        lg = np.empty(self.V, np.float32)
        rc = self.xr.lib.xref_decode_step(self.h, int(tok), lg.ctypes.data)
        if rc:
            raise RuntimeError(f"xref_decode_step rc={rc}")
        return lg

    def prefill(self, toks, all_logits=True):
        toks = np.ascontiguousarray(toks, np.int32)
        lg = np.empty((toks.size, self.V), np.float32) if all_logits else None
        rc = self.xr.lib.xref_prefill(self.h, toks.ctypes.data, toks.size,
                                      lg.ctypes.data if all_logits else None)
        if rc:
            raise RuntimeError(f"xref_prefill rc={rc}")
        return lg

    def rewind(self, n):
        return self.xr.lib.xref_rewind(self.h, n)

    def position(self):
        return self.xr.lib.xref_position(self.h)

    def clone(self):
        h = C.c_void_p()
        rc = self.xr.lib.xref_clone(self.h, C.byref(h))
        if rc:
            raise RuntimeError(f"xref_clone rc={rc}")
        return XrefSession(self.xr, self.desc, self.max_ctx, handle=h, flags=self.flags)

    def kv_bytes(self, layer, pos, which):
        """Spinor sessions: the cached blocks of one layer at one position."""
        c = self.desc.cfg
        o = np.zeros(c.n_head_kv * self.xr.spinor_blocks_for(c.head_dim) * 63, np.uint8)
        rc = self.xr.lib.xref_kv_bytes(self.h, layer, pos, which, o.ctypes.data)
        if rc:
            raise RuntimeError(f"xref_kv_bytes rc={rc}")
        return o

    def kv(self, layer, pos, which):
        c = self.desc.cfg
        o = np.empty(c.n_head_kv * c.head_dim, np.int32)
        self.xr.lib.xref_kv_read(self.h, layer, pos, which, o.ctypes.data)
        return o


# ----------------------------------------------------------------------------- reference
class RefLib:
    """The reference's compiled L1 library (float forward, session ABI, islands)."""

    def __init__(self, path=SPREF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = L = C.CDLL(path)
        L.sp_model_load.argtypes = [C.c_char_p, C.c_char_p, C.POINTER(C.c_void_p)]
        L.sp_model_unload.argtypes = [C.c_void_p]
        L.sp_session_create.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]
        L.sp_session_destroy.argtypes = [C.c_void_p]
        L.sp_prefill_chunk.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]
        L.sp_decode_step.argtypes = [C.c_void_p, C.c_int32, C.c_void_p, C.c_size_t]
        L.sp_session_clone.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]
        L.sp_session_rewind.argtypes = [C.c_void_p, C.c_size_t]
        L.sp_session_position.argtypes = [C.c_void_p, C.POINTER(C.c_size_t)]
        L.sp_session_register_forward_backend.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
        L.sp_session_register_kvdecode_backend.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
        L.sp_session_qwen3_model.argtypes = [C.c_void_p]
        L.sp_session_qwen3_model.restype = C.c_void_p
        L.sp_last_error.restype = C.c_char_p
        L.sp_xxh64.argtypes = [C.c_void_p, C.c_size_t, C.c_uint64]
        L.sp_xxh64.restype = C.c_uint64
        L.sp_crc32.argtypes = [C.c_void_p, C.c_size_t]
        L.sp_crc32.restype = C.c_uint32
        for f in ("sp_rmsnorm_exact",):
            getattr(L, f).argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.sp_softmax_exact.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.sp_gelu_exact.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.sp_f16_to_f32.argtypes = [C.c_uint16]
        L.sp_f16_to_f32.restype = C.c_float
        L.sp_frob_quant1.argtypes = [C.c_float, C.c_float]
        L.sp_frob_quant1.restype = C.c_int8

    def err(self):
        e = self.lib.sp_last_error()
        return e.decode() if e else ""

    def load(self, model_path, tok_path):
        m = C.c_void_p()
        rc = self.lib.sp_model_load(model_path.encode(), tok_path.encode(), C.byref(m))
        if rc:
            raise RuntimeError(f"sp_model_load rc={rc}: {self.err()}")
        return m

    def session(self, model, max_ctx=0):
        cfg = (C.c_byte * 64)()          # sp_session_config, zeroed; max_context first
        C.c_size_t.from_buffer(cfg, 0).value = max_ctx
        s = C.c_void_p()
        rc = self.lib.sp_session_create(model, cfg, None, C.byref(s))
        if rc:
            raise RuntimeError(f"sp_session_create rc={rc}: {self.err()}")
        return s

    def prefill(self, s, toks, V):
        toks = np.ascontiguousarray(toks, np.int32)
        lg = np.empty(V, np.float32)
        rc = self.lib.sp_prefill_chunk(s, toks.ctypes.data, toks.size, lg.ctypes.data, V)
        return rc, lg

    def decode(self, s, tok, V):
        lg = np.empty(V, np.float32)
        rc = self.lib.sp_decode_step(s, int(tok), lg.ctypes.data, V)
        return rc, lg

    def position(self, s):
        p = C.c_size_t()
        self.lib.sp_session_position(s, C.byref(p))
        return p.value
