"""ctypes bindings of libspb200.so / libspb200_l1.so (include/spb200.h, spb200_l1.h).

The host-side mirror of the reference's L1 interface for this path, used by the tests
and bench.py: plain pointers in, status codes out, the library's own error text in
`SpbError`. There is no fallback: if the CUDA library cannot be loaded, `load()` raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
CORE_SO = os.path.join(HERE, "libspb200.so")
L1_SO = os.path.join(HERE, "libspb200_l1.so")

SPB_OK, SPB_ENOMEM, SPB_EBADARG, SPB_EBADSTATE = 0, -1, -3, -4
SPB_EUNSUPPORTED, SPB_ECONTEXT_FULL, SPB_ECUDA, SPB_EOOM, SPB_ERANGE = -5, -33, -40, -43, -50
SPB_KV_SPINOR = 1   # spb_session_open_ex flag: K/V rows as Spinor blocks

# symbols include/spb200.h declares (checked by the CPU test suite)
CORE_SYMBOLS = [
    "spb_last_error", "spb_device_count", "spb_model_upload", "spb_model_synthetic", "spb_model_free",
    "spb_model_weight_bytes", "spb_session_open", "spb_session_prefill", "spb_session_decode_step",
    "spb_session_decode_step_argmax", "spb_session_decode_greedy", "spb_session_rewind",
    "spb_session_position", "spb_session_clone", "spb_session_close", "spb_session_kv_read",
    "spb_session_stream", "spb_forward", "spb_gemv_q4b", "spb_gemv_q4b_noalloc", "spb_quantize_rows",
    "spb_gemv_q4b_q",
    "spb_gemv_q4b_gated_q", "spb_rmsnorm_exact_dev", "spb_gelu_exact_dev",
    "spb_silu_exact_dev", "spb_rope_cordic_dev", "spb_take_device_errors", "spb_rope_freq_table",
    "spb_cordic_tables", "spb_graph_begin", "spb_graph_end", "spb_graph_launch", "spb_graph_free",
    "spb_batch_decode_step", "spb_q4b_prepare", "spb_q4b_release", "spb_q4b_info", "spb_q4b_matmul",
    "spb_tp_shard", "spb_tp_unique_id", "spb_tp_open", "spb_tp_close", "spb_tp_rank", "spb_tp_world",
    "spb_model_synthetic_tp", "spb_model_upload_tp", "spb_tp_p2p_init", "spb_tp_p2p_connect",
    "spb_tp_p2p_loopback", "spb_kvpool_create", "spb_kvpool_free", "spb_kvpool_free_pages",
    "spb_session_open_paged", "spb_session_open_ex", "spb_session_kv_bytes",
]
L1_SYMBOLS = ["spb_l1_forward", "spb_l1_backend", "spb_l1_kvdecode_table", "spb_l1_kvdecode_clone",
              "spb_l1_set_device", "spb_l1_release_model", "spb_l1_kvdecode_table_ext", "spb_l1_set_kv_pool",
              "spb_l1_set_kv_flags"]


class SpbError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"spb rc={code}: {msg}")
        self.code = code


class Q4B(C.Structure):
    _fields_ = [("codes", C.c_void_p), ("bscale", C.c_void_p), ("rows", C.c_int32), ("cols", C.c_int32)]


class LayerDesc(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("attn_norm", "q_norm", "k_norm", "post_attn_norm",
                                          "ffn_norm", "post_ffw_norm")] + \
               [(n, Q4B) for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd")]


class Config(C.Structure):
    _fields_ = [("arch", C.c_int32), ("n_layers", C.c_int32), ("n_embd", C.c_int32),
                ("n_ff", C.c_int32), ("n_head", C.c_int32), ("n_head_kv", C.c_int32),
                ("head_dim", C.c_int32), ("n_vocab", C.c_int32), ("sliding_window", C.c_int32),
                ("rope_base", C.c_float), ("rope_base_local", C.c_float),
                ("swa_period", C.c_int32), ("has_qk_norm", C.c_int32)]


class ModelDesc(C.Structure):
    _fields_ = [("cfg", Config), ("layers", C.c_void_p), ("token_embd", Q4B),
                ("output", Q4B), ("output_norm", C.c_void_p)]


_LAYER_MAP = [("attn_norm", "attn_norm"), ("q_norm", "attn_q_norm"), ("k_norm", "attn_k_norm"),
              ("post_attn_norm", "post_attention_norm"), ("ffn_norm", "ffn_norm"),
              ("post_ffw_norm", "post_ffw_norm")]
_MAT_MAP = [("wq", "attn_q"), ("wk", "attn_k"), ("wv", "attn_v"), ("wo", "attn_output"),
            ("wg", "ffn_gate"), ("wu", "ffn_up"), ("wd", "ffn_down")]


def _ptr(a):
    return None if a is None else a.ctypes.data


def config_struct(cfg) -> Config:
    return Config(cfg.arch, cfg.n_layers, cfg.n_embd, cfg.n_ff, cfg.n_head, cfg.n_head_kv,
                  cfg.head_dim, cfg.n_vocab, cfg.sliding_window, cfg.rope_base,
                  cfg.rope_base_local, cfg.swa_period, cfg.has_qk_norm)


def model_desc(cfg, T) -> ModelDesc:
    """Descriptor over the host tensors of spmodel.gen_model (keeps them alive)."""
    layers = (LayerDesc * cfg.n_layers)()
    for L in range(cfg.n_layers):
        ly = layers[L]
        for f, nm in _LAYER_MAP:
            setattr(ly, f, _ptr(T.get(f"blk.{L}.{nm}.weight")))
        for f, nm in _MAT_MAP:
            t = T[f"blk.{L}.{nm}.weight"]
            setattr(ly, f, Q4B(_ptr(t.codes), _ptr(t.bscale), t.rows, t.cols))
    emb = T["token_embd.weight"]
    out = T.get("output.weight", emb)
    m = ModelDesc(config_struct(cfg), C.addressof(layers),
                  Q4B(_ptr(emb.codes), _ptr(emb.bscale), emb.rows, emb.cols),
                  Q4B(_ptr(out.codes), _ptr(out.bscale), out.rows, out.cols),
                  _ptr(T["output_norm.weight"]))
    m._keep = (layers, T)
    return m


_lib = None


def load(path: str = CORE_SO):
    """Load libspb200.so (raises if it is missing: there is no CPU fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} not built (run shannon-prime-system_b200/build.py)")
    L = C.CDLL(path)
    vp, i32, i64 = C.c_void_p, C.c_int32, C.c_int64
    sig = {
        "spb_last_error": ([], C.c_char_p), "spb_device_count": ([], C.c_int),
        "spb_model_upload": ([vp, C.c_int, C.POINTER(vp)], C.c_int),
        "spb_model_synthetic": ([vp, C.c_uint64, C.c_int, C.POINTER(vp)], C.c_int),
        "spb_model_free": ([vp], None), "spb_model_weight_bytes": ([vp], i64),
        "spb_session_open": ([vp, C.c_int, C.POINTER(vp)], C.c_int),
        "spb_session_prefill": ([vp, vp, C.c_int, vp], C.c_int),
        "spb_session_decode_step": ([vp, i32, vp], C.c_int),
        "spb_session_decode_step_argmax": ([vp, i32, vp, vp], C.c_int),
        "spb_session_decode_greedy": ([vp, i32, C.c_int, vp], C.c_int),
        "spb_batch_decode_step": ([vp, C.c_int, vp, vp, vp], C.c_int),
        "spb_session_rewind": ([vp, C.c_int], C.c_int), "spb_session_position": ([vp], C.c_int),
        "spb_session_clone": ([vp, C.POINTER(vp)], C.c_int), "spb_session_close": ([vp], None),
        "spb_session_kv_read": ([vp, C.c_int, C.c_int, C.c_int, vp], C.c_int),
        "spb_session_stream": ([vp], vp),
        "spb_forward": ([vp, vp, C.c_int, vp], C.c_int),
        "spb_gemv_q4b": ([vp, vp, C.c_int, C.c_int, vp, C.c_int, vp, vp], C.c_int),
        "spb_gemv_q4b_noalloc": ([vp, vp, C.c_int, C.c_int, vp, C.c_int, vp, vp], C.c_int),
        "spb_q4b_prepare": ([vp, vp, C.c_int, C.c_int, vp, C.POINTER(vp)], C.c_int),
        "spb_tp_p2p_loopback": ([C.c_int, C.c_uint32, C.c_int, C.c_int], C.c_int),
        "spb_kvpool_create": ([vp, C.c_int, C.c_int, C.POINTER(vp)], C.c_int),
        "spb_kvpool_free": ([vp], None), "spb_kvpool_free_pages": ([vp], C.c_int),
        "spb_session_open_paged": ([vp, C.c_int, C.POINTER(vp)], C.c_int),
        "spb_session_open_ex": ([vp, C.c_int, C.c_uint, C.POINTER(vp)], C.c_int),
        "spb_session_kv_bytes": ([vp, C.c_int, C.c_int, C.c_int, vp], C.c_int),
        "spb_q4b_release": ([vp], None),
        "spb_q4b_info": ([vp, vp], C.c_int),
        "spb_q4b_matmul": ([vp, vp, C.c_int, vp, vp], C.c_int),
        "spb_quantize_rows": ([vp, C.c_int, C.c_int, vp, vp, vp, vp], C.c_int),
        "spb_gemv_q4b_q": ([vp, vp, C.c_int, C.c_int, vp, vp, vp, C.c_int, vp, vp], C.c_int),
        "spb_gemv_q4b_gated_q": ([vp, vp, vp, vp, C.c_int, C.c_int, vp, vp, vp, C.c_int, C.c_int, vp, vp],
                                 C.c_int),
        "spb_rmsnorm_exact_dev": ([vp, vp, C.c_int, C.c_int, vp, vp], C.c_int),
        "spb_gelu_exact_dev": ([vp, C.c_int, vp, vp], C.c_int),
        "spb_silu_exact_dev": ([vp, C.c_int, vp, vp], C.c_int),
        "spb_rope_cordic_dev": ([vp, C.c_int, C.c_int, vp, C.c_float, vp, vp], C.c_int),
        "spb_take_device_errors": ([], C.c_int),
        "spb_rope_freq_table": ([C.c_float, C.c_int, vp], C.c_int),
        "spb_cordic_tables": ([vp, vp], None),
        "spb_graph_begin": ([vp], C.c_int), "spb_graph_end": ([vp, C.POINTER(vp)], C.c_int),
        "spb_graph_launch": ([vp, vp], C.c_int), "spb_graph_free": ([vp], None),
        "spb_tp_shard": ([vp, C.c_int, C.c_int, vp], C.c_int),
        "spb_tp_unique_id": ([vp], C.c_int),
        "spb_tp_open": ([vp, C.c_int, C.c_int, C.c_int, C.POINTER(vp)], C.c_int),
        "spb_tp_close": ([vp], None), "spb_tp_rank": ([vp], C.c_int), "spb_tp_world": ([vp], C.c_int),
        "spb_model_synthetic_tp": ([vp, C.c_uint64, vp, C.POINTER(vp)], C.c_int),
        "spb_model_upload_tp": ([vp, vp, C.POINTER(vp)], C.c_int),
        "spb_tp_p2p_init": ([vp, C.c_int, vp], C.c_int), "spb_tp_p2p_connect": ([vp, vp], C.c_int),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


def check(rc):
    if rc != SPB_OK:
        raise SpbError(rc, (load().spb_last_error() or b"").decode())
    return rc


def rope_table(base, d):
    W = np.zeros(d // 2, np.uint64)
    check(load().spb_rope_freq_table(base, d, W.ctypes.data))
    return W


def cordic_tables():
    T = np.zeros(30, np.uint64)
    g = C.c_uint64()
    load().spb_cordic_tables(T.ctypes.data, C.byref(g))
    return T, g.value


TP_ID_BYTES = 128
TP_P2P_BLOB_BYTES = 80


def tp_shard(cfg, rank, world):
    """(h0, nh, kv0, nkv, f0, nff, v0, nv): rank's query heads, KV heads, FFN columns and
    LM-head rows (host only)."""
    c = config_struct(cfg)
    out = np.zeros(8, np.int32)
    check(load().spb_tp_shard(C.byref(c), rank, world, out.ctypes.data))
    return tuple(int(v) for v in out)


def tp_unique_id():
    b = (C.c_uint8 * TP_ID_BYTES)()
    check(load().spb_tp_unique_id(b))
    return bytes(b)


def tp_uid_from_dist(group=None):
    """The group's unique id on every rank of the current torch.distributed group: rank 0 makes
    it, a broadcast shares it (any backend; host only)."""
    import torch.distributed as dist
    obj = [tp_unique_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


class TensorParallel:
    """One rank of a tensor-parallel group (one process per GPU); every rank opens it with the
    same unique id (from tp_unique_id on one rank, shared by the caller)."""

    def __init__(self, uid: bytes, rank, world, device):
        if len(uid) != TP_ID_BYTES:
            raise ValueError("unique id must be 128 bytes")
        b = (C.c_uint8 * TP_ID_BYTES).from_buffer_copy(uid)
        self.h = C.c_void_p()
        check(load().spb_tp_open(b, rank, world, device, C.byref(self.h)))
        self.rank, self.world, self.device = rank, world, device

    def enable_p2p(self, cap, group=None):
        """Collective: exchanges of at most `cap` values (the decode step's) run over peer
        memory instead of NCCL; the mailbox handles travel over the torch.distributed group."""
        import torch.distributed as dist
        blob = (C.c_uint8 * TP_P2P_BLOB_BYTES)()
        check(load().spb_tp_p2p_init(self.h, cap, blob))
        blobs = [None] * self.world
        dist.all_gather_object(blobs, bytes(blob), group=group)
        allb = (C.c_uint8 * (TP_P2P_BLOB_BYTES * self.world)).from_buffer_copy(b"".join(blobs))
        check(load().spb_tp_p2p_connect(self.h, allb))

    def close(self):
        if self.h:
            load().spb_tp_close(self.h)
            self.h = None


class Model:
    def __init__(self, handle, cfg):
        self.h, self.cfg = handle, cfg

    @classmethod
    def upload_tp(cls, cfg, T, tp):
        """This rank's shard of a whole host model (logits and argmax stay full-vocabulary)."""
        d = model_desc(cfg, T)
        h = C.c_void_p()
        check(load().spb_model_upload_tp(C.byref(d), tp.h, C.byref(h)))
        return cls(h, cfg)

    @classmethod
    def synthetic_tp(cls, cfg, tp, seed=0):
        c = config_struct(cfg)
        h = C.c_void_p()
        check(load().spb_model_synthetic_tp(C.byref(c), seed, tp.h, C.byref(h)))
        return cls(h, cfg)

    @classmethod
    def upload(cls, cfg, T, device=0):
        d = model_desc(cfg, T)
        h = C.c_void_p()
        check(load().spb_model_upload(C.byref(d), device, C.byref(h)))
        return cls(h, cfg)

    @classmethod
    def synthetic(cls, cfg, seed=0, device=0):
        c = config_struct(cfg)
        h = C.c_void_p()
        check(load().spb_model_synthetic(C.byref(c), seed, device, C.byref(h)))
        return cls(h, cfg)

    def weight_bytes(self):
        return load().spb_model_weight_bytes(self.h)

    def forward(self, tokens):
        tokens = np.ascontiguousarray(tokens, np.int32)
        lg = np.empty((tokens.size, self.cfg.n_vocab), np.float32)
        check(load().spb_forward(self.h, tokens.ctypes.data, tokens.size, lg.ctypes.data))
        return lg

    def session(self, pmax, spinor=False):
        """A resident-KV session; spinor=True keeps K/V as Spinor blocks (SPB_KV_SPINOR)."""
        return Session(self, pmax, flags=SPB_KV_SPINOR if spinor else 0)

    def free(self):
        if self.h:
            load().spb_model_free(self.h)
            self.h = None


class KvPool:
    """A pool of paged, copy-on-write K/V pages on the model's device (spb_kvpool_create)."""

    def __init__(self, model, page_positions, n_pages):
        h = C.c_void_p()
        check(load().spb_kvpool_create(model.h, page_positions, n_pages, C.byref(h)))
        self.h, self.model, self.pg, self.n_pages = h, model, page_positions, n_pages

    def session(self, pmax):
        h = C.c_void_p()
        check(load().spb_session_open_paged(self.h, pmax, C.byref(h)))
        return Session(self.model, pmax, handle=h)

    def free_pages(self):
        return load().spb_kvpool_free_pages(self.h)

    def free(self):
        if self.h:
            load().spb_kvpool_free(self.h)
            self.h = None


class Session:
    def __init__(self, model, pmax, handle=None, flags=0):
        self.model, self.pmax, self.flags = model, pmax, flags
        self.V = model.cfg.n_vocab
        if handle is None:
            handle = C.c_void_p()
            check(load().spb_session_open_ex(model.h, pmax, flags, C.byref(handle)))
        self.h = handle

    def prefill(self, tokens, logits=True):
        tokens = np.ascontiguousarray(tokens, np.int32)
        lg = np.empty((tokens.size, self.V), np.float32) if logits else None
        check(load().spb_session_prefill(self.h, tokens.ctypes.data, tokens.size,
                                         lg.ctypes.data if logits else None))
        return lg

    def step(self, token, out=None):
        lg = out if out is not None else np.empty(self.V, np.float32)
        check(load().spb_session_decode_step(self.h, int(token), lg.ctypes.data))
        return lg

    def step_argmax(self, token, out=None):
        lg = out if out is not None else np.empty(self.V, np.float32)
        am = C.c_int32()
        check(load().spb_session_decode_step_argmax(self.h, int(token), lg.ctypes.data, C.byref(am)))
        return lg, am.value

    def greedy(self, token, n):
        out = np.empty(n, np.int32)
        check(load().spb_session_decode_greedy(self.h, int(token), n, out.ctypes.data))
        return out

    def rewind(self, n):
        check(load().spb_session_rewind(self.h, n))

    def position(self):
        return load().spb_session_position(self.h)

    def clone(self):
        h = C.c_void_p()
        check(load().spb_session_clone(self.h, C.byref(h)))
        return Session(self.model, self.pmax, handle=h, flags=self.flags)

    def kv(self, layer, pos, which):
        c = self.model.cfg
        o = np.empty(c.n_head_kv * c.head_dim, np.int32)
        check(load().spb_session_kv_read(self.h, layer, pos, which, o.ctypes.data))
        return o

    def kv_bytes(self, layer, pos, which):
        """A Spinor session's cached blocks of one layer and position (uint8)."""
        c = self.model.cfg
        nb = 1 if c.head_dim <= 55 else (c.head_dim + 54) // 55
        o = np.empty(c.n_head_kv * nb * 63, np.uint8)
        check(load().spb_session_kv_bytes(self.h, layer, pos, which, o.ctypes.data))
        return o

    def stream(self):
        return load().spb_session_stream(self.h)

    def close(self):
        if self.h:
            load().spb_session_close(self.h)
            self.h = None


def batch_decode(sessions, tokens, logits=True):
    """One decode step for several sessions at once (spb_batch_decode_step): returns
    (logits [B][V] or None, argmax [B])."""
    B = len(sessions)
    hs = (C.c_void_p * B)(*[s.h for s in sessions])
    tok = np.ascontiguousarray(np.asarray(tokens, np.int32))
    V = sessions[0].V
    lg = np.empty((B, V), np.float32) if logits else None
    am = np.empty(B, np.int32)
    check(load().spb_batch_decode_step(hs, B, tok.ctypes.data, lg.ctypes.data if logits else None,
                                       am.ctypes.data))
    return lg, am


class PreparedQ4B:
    """An OK_Q4B matrix already in device memory, prepared once (spb_q4b_prepare: the exact-range
    check and the block-scale description); matmul takes any number of token rows. Pointers are
    device addresses (ints or c_void_p); the codes and scales must outlive the handle."""

    def __init__(self, codes, bscale, rows, cols, stream=None):
        h = C.c_void_p()
        check(load().spb_q4b_prepare(codes, bscale, rows, cols, stream, C.byref(h)))
        self.h, self.rows, self.cols = h, rows, cols

    def info(self):
        o = (C.c_int32 * 4)()
        check(load().spb_q4b_info(self.h, o))
        return {"rows": o[0], "cols": o[1], "small": o[2], "planes": o[3]}

    def matmul(self, x, n_tok, y, stream=None):
        check(load().spb_q4b_matmul(self.h, x, n_tok, y, stream))

    def release(self):
        if self.h:
            load().spb_q4b_release(self.h)
            self.h = None


def load_l1(path: str = L1_SO):
    """The section-6/6b binding; the reference L1 library must already be loaded
    RTLD_GLOBAL in this process (it provides sp_arena_find / sp_as_f32 / sp_set_error)."""
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} not built")
    L = C.CDLL(path, mode=C.RTLD_GLOBAL)
    L.spb_l1_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
    L.spb_l1_forward.restype = C.c_int
    L.spb_l1_backend.restype = C.c_void_p
    L.spb_l1_kvdecode_table.restype = C.c_void_p
    L.spb_l1_kvdecode_clone.argtypes = [C.c_void_p, C.POINTER(C.c_void_p)]
    L.spb_l1_set_device.argtypes = [C.c_int]
    L.spb_l1_release_model.argtypes = [C.c_void_p]
    L.spb_l1_kvdecode_table_ext.restype = C.c_void_p
    L.spb_l1_set_kv_pool.argtypes = [C.c_int, C.c_int]
    return L
