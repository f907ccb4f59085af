"""Seeded synthetic OK_Q4B models and the `.sp-model` / `.sp-tokenizer` writer.

The reference loads models only from `.sp-model` files (sp_model.h:83-118, loader
sp_model_load.c:119-186, Q4B reconstruction sp_model_bridge.c:114-148). This module
writes such files for synthetic random-init models so the reference's own session
(and therefore the section-6 / section-6b backends) can be driven on the configs
the benchmarks name, and it hands the same tensors to the C-ABI as plain pointers.

Generator (counter-based, identical on host and device -- see spb_synth_fill in the
CUDA library): every tensor owns a stream id; word(seed, stream, i) is a 64-bit
splitmix64 hash, so any element can be produced independently.
  * codes   : byte j of a Q4B matrix = byte (j % 8) of word(seed, stream, j // 8)
              -> every nibble uniform over all 16 values (-8..7)
  * bscale  : f16 with exponent e = floor(log2(1 / (8 * sqrt(cols)))), a uniform random
              10-bit mantissa and a random sign (bit 10 of the word), i.e. +-uniform in
              [2^e, 2^(e+1)). The sign matters: uniform nibbles have mean -1/2, so with
              positive scales every row shares a common-mode component, the gate and up
              products share it too, and a model without sandwich norms (Qwen3) carries a
              coherent offset into its residual stream that leaves the exact range within
              three layers at the 8B width; random signs remove the common mode
  * norms   : (7549747 + (word >> 40) % 1677722) * 2^-23, i.e. in [0.9, 1.1)
  * tokens  : word % n_vocab
"""
from __future__ import annotations

import dataclasses
import hashlib
import math
import struct
import zlib

import numpy as np

M64 = (1 << 64) - 1


# ----------------------------------------------------------------------------- configs
@dataclasses.dataclass(frozen=True)
class Config:
    name: str
    arch: int                 # 0 = qwen3, 1 = gemma3 (the descriptor's arch field)
    n_layers: int
    n_embd: int
    n_ff: int
    n_head: int
    n_head_kv: int
    head_dim: int
    n_vocab: int
    sliding_window: int = 0
    rope_base: float = 1e6
    rope_base_local: float = 10000.0
    swa_period: int = 6
    has_qk_norm: int = 1
    max_context: int = 4096

    @property
    def gemma(self) -> bool:
        return self.arch == 1

    @property
    def qd(self) -> int:
        return self.n_head * self.head_dim

    @property
    def kvd(self) -> int:
        return self.n_head_kv * self.head_dim

    def weight_bytes(self) -> int:
        """HBM bytes of all OK_Q4B matrices streamed by one decode token."""
        def q4b(rows, cols):
            return rows * (cols // 2) + rows * ((cols + 31) // 32) * 2
        E, FF = self.n_embd, self.n_ff
        per = (q4b(self.qd, E) + 2 * q4b(self.kvd, E) + q4b(E, self.qd)
               + 2 * q4b(FF, E) + q4b(E, FF))
        return self.n_layers * per + q4b(self.n_vocab, E)


ARCH_QWEN3, ARCH_GEMMA3 = 0, 1

CONFIGS = {
    # tiny Gemma-style decoder (reference-CPU runnable)
    "tiny": Config("tiny", ARCH_GEMMA3, 4, 512, 2048, 8, 2, 64, 8192,
                   sliding_window=512, rope_base=1e6, max_context=256),
    # Gemma-3-12B shape
    "gemma12b": Config("gemma12b", ARCH_GEMMA3, 48, 3840, 15360, 16, 8, 256, 262144,
                       sliding_window=1024, rope_base=1e6, max_context=4096),
    # Qwen3-8B shape
    "qwen8b": Config("qwen8b", ARCH_QWEN3, 36, 4096, 12288, 32, 8, 128, 151936,
                     rope_base=1e6, max_context=8192),
    # small parity shapes (CPU-checkable in seconds)
    "micro_gemma": Config("micro_gemma", ARCH_GEMMA3, 7, 256, 512, 4, 2, 64, 1024,
                          sliding_window=16, rope_base=1e6, max_context=128),
    "micro_qwen": Config("micro_qwen", ARCH_QWEN3, 3, 256, 768, 8, 2, 64, 1024,
                         rope_base=1e6, max_context=128),
}


def derive(cfg: Config, **kw) -> Config:
    return dataclasses.replace(cfg, **kw)


# ----------------------------------------------------------------------------- RNG
def _splitmix64(z):
    z = (z + np.uint64(0x9E3779B97F4A7C15)) & np.uint64(M64)
    z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & np.uint64(M64)
    z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & np.uint64(M64)
    return z ^ (z >> np.uint64(31))


def stream_key(seed: int, stream: int) -> int:
    with np.errstate(over="ignore"):
        return int(_splitmix64(np.uint64(((seed & M64) * 0x10001 + stream) & M64)))


def words(seed: int, stream: int, n: int, start: int = 0) -> np.ndarray:
    key = np.uint64(stream_key(seed, stream))
    with np.errstate(over="ignore"):
        idx = np.arange(start, start + n, dtype=np.uint64)
        return _splitmix64(idx + key)


def scale_exponent(cols: int) -> int:
    return math.floor(math.log2(1.0 / (8.0 * math.sqrt(cols))))


def gen_codes(seed, stream, rows, cols):
    nib = (cols + 1) // 2
    nbytes = rows * nib
    w = words(seed, stream, (nbytes + 7) // 8)
    return w.view(np.uint8)[:nbytes].reshape(rows, nib).copy()


def gen_bscale(seed, stream, rows, cols):
    nblk = (cols + 31) // 32
    e = scale_exponent(cols)
    w = words(seed, stream, rows * nblk)
    bits = (np.uint64((e + 15) << 10) | (w & np.uint64(0x3FF)) |
            (((w >> np.uint64(10)) & np.uint64(1)) << np.uint64(15))).astype(np.uint16)
    return bits.reshape(rows, nblk)


def gen_norm(seed, stream, n):
    w = words(seed, stream, n)
    k = np.uint64(7549747) + (w >> np.uint64(40)) % np.uint64(1677722)
    return (k.astype(np.float64) * 2.0 ** -23).astype(np.float32)


def gen_tokens(seed, n, n_vocab, stream=7):
    return (words(seed, stream, n) % np.uint64(n_vocab)).astype(np.int32)


# tensor -> stream ids (matrices: codes use 2*id, scales 2*id + 1)
GLOBAL_IDS = {"token_embd.weight": 1, "output.weight": 2, "output_norm.weight": 3}
LAYER_FIELDS = ["attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "attn_q_norm",
                "attn_k_norm", "post_attention_norm", "ffn_norm", "ffn_gate", "ffn_up",
                "ffn_down", "post_ffw_norm"]


def tensor_id(name: str) -> int:
    if name in GLOBAL_IDS:
        return GLOBAL_IDS[name]
    _, L, field, _ = name.split(".")
    return 64 + 64 * int(L) + LAYER_FIELDS.index(field)


@dataclasses.dataclass
class Q4B:
    codes: np.ndarray    # uint8 [rows][ceil(cols/2)]
    bscale: np.ndarray   # uint16 [rows][ceil(cols/32)]
    rows: int
    cols: int


def layer_shapes(cfg: Config):
    E, FF = cfg.n_embd, cfg.n_ff
    return {"attn_q": (cfg.qd, E), "attn_k": (cfg.kvd, E), "attn_v": (cfg.kvd, E),
            "attn_output": (E, cfg.qd), "ffn_gate": (FF, E), "ffn_up": (FF, E),
            "ffn_down": (E, FF)}


def layer_norms(cfg: Config):
    n = {"attn_norm": cfg.n_embd, "ffn_norm": cfg.n_embd,
         "attn_q_norm": cfg.head_dim, "attn_k_norm": cfg.head_dim}
    if cfg.gemma:
        n["post_attention_norm"] = cfg.n_embd
        n["post_ffw_norm"] = cfg.n_embd
    return n


def gen_matrix(seed, name, rows, cols) -> Q4B:
    tid = tensor_id(name)
    return Q4B(gen_codes(seed, 2 * tid, rows, cols), gen_bscale(seed, 2 * tid + 1, rows, cols),
               rows, cols)


# ----------------------------------------------------------------------------- adversarial scales
# The exact int64 accumulation bound every row must keep (the checker's xref_q4b_check and the
# library's upload/prepare test): sum_b |k_b| * 32 * 8 * 127 < 2^63, k_b the f16 scale * 2^24.
BOUND_LIMIT = (1 << 63) // (32 * 8 * 127)


def f16_k(h: int) -> int:
    """The f16 bit pattern h as the integer k = value * 2^24 (finite values only)."""
    e, m = (h >> 10) & 31, h & 1023
    k = m if e == 0 else (1024 | m) << (e - 1)
    return -k if h & 0x8000 else k


def k_to_f16(k: int) -> int:
    """The f16 bits of the value k * 2^-24, for a k that f16 represents exactly."""
    neg, k = k < 0, abs(k)
    if k < 1024:
        h = k
    else:
        sh = k.bit_length() - 11
        assert k == (k >> sh) << sh and 0 <= sh <= 29, k
        h = ((sh + 1) << 10) | ((k >> sh) & 1023)
    return h | (0x8000 if neg else 0)


def adversarial_bscale(seed: int, rows: int, cols: int, kind: str) -> np.ndarray:
    """Block scales that the seeded generator never makes, row-major [rows][cols/32] f16 bits:
      signs     random signs, one exponent per row (spread 0), a few zero and subnormal blocks
      large     |scale| >= 128 (exponent fields 22-23): outside the token-batch GEMM's small form
      spreadN   exponent fields vary within a row by up to N (N = 1, 9, 17), random signs
      full      exponent fields 0-30 within a row (subnormal to the f16 maximum), random signs
    Rows whose sum would break the exact bound have their largest blocks lowered until it holds."""
    rng = np.random.default_rng(seed)
    nblk = cols // 32
    mant = rng.integers(0, 1024, (rows, nblk))
    sign = rng.integers(0, 2, (rows, nblk)) << 15
    if kind == "signs":
        base = rng.integers(4, 12, (rows, 1))
        e = np.broadcast_to(base, (rows, nblk)).copy()
        z = rng.random((rows, nblk))
        e[z < 0.05] = 0                               # subnormal (mantissa may be 0: a zero block)
        mant[z < 0.02] = 0
        if rows > 1:
            e[1], mant[1] = 0, 0                      # an all-zero row
    elif kind == "large":
        e = rng.integers(22, 24, (rows, nblk))
    elif kind.startswith("spread"):
        n = int(kind[6:])
        lo = rng.integers(1, 30 - n, (rows, 1))
        e = lo + rng.integers(0, n + 1, (rows, nblk))
    elif kind == "full":
        e = rng.integers(0, 31, (rows, nblk))
    else:
        raise ValueError(kind)
    h = ((e.astype(np.int64) << 10) | mant | sign).astype(np.uint16)
    for r in range(rows):   # keep every row inside the bound
        while sum(abs(f16_k(int(x))) for x in h[r]) >= BOUND_LIMIT:
            b = int(np.argmax((h[r] >> 10) & 31))
            h[r, b] = np.uint16(int(h[r, b]) - (1 << 10))
    return h


def model_bscale(seed: int, rows: int, cols: int, spread: int) -> np.ndarray:
    """Block scales for whole-model tests: the seeded generator's magnitude (its exponent for
    `cols` is the largest), lowered per block by 0..spread exponent steps (down to subnormal),
    random signs and 3 % zero blocks, so activations keep the exact range."""
    rng = np.random.default_rng(seed)
    nblk = cols // 32
    e = np.maximum(scale_exponent(cols) + 15 - rng.integers(0, spread + 1, (rows, nblk)), 0)
    mant = rng.integers(0, 1024, (rows, nblk))
    mant[rng.random((rows, nblk)) < 0.03] = 0
    mant[e == 0] |= 0            # subnormal blocks keep their mantissa (value mant * 2^-24)
    e = np.where(mant == 0, 0, e)
    sign = rng.integers(0, 2, (rows, nblk)) << 15
    return ((e.astype(np.int64) << 10) | mant | sign).astype(np.uint16)


def bound_edge_row(nblk: int, total: int) -> np.ndarray:
    """One row of nblk positive block scales whose integers k sum to exactly `total` (as many
    f16-maximum blocks as fit, then the remainder greedily), for the bound's edge cases."""
    kmax = 2047 << 29
    out = []
    r = total
    while r > 0:
        if r >= kmax:
            k = kmax
        elif r < 1024:
            k = r
        else:
            sh = r.bit_length() - 11
            k = (r >> sh) << sh
        out.append(k_to_f16(k))
        r -= k
    assert len(out) <= nblk, (len(out), nblk)
    return np.array(out + [0] * (nblk - len(out)), np.uint16)


def gen_model(cfg: Config, seed: int = 0) -> dict:
    """All tensors of a random-init model, keyed by their .sp-model names."""
    T = {}
    T["token_embd.weight"] = gen_matrix(seed, "token_embd.weight", cfg.n_vocab, cfg.n_embd)
    if not cfg.gemma:
        T["output.weight"] = gen_matrix(seed, "output.weight", cfg.n_vocab, cfg.n_embd)
    T["output_norm.weight"] = gen_norm(seed, 2 * tensor_id("output_norm.weight"), cfg.n_embd)
    for L in range(cfg.n_layers):
        for f, (r, c) in layer_shapes(cfg).items():
            nm = f"blk.{L}.{f}.weight"
            T[nm] = gen_matrix(seed, nm, r, c)
        for f, n in layer_norms(cfg).items():
            nm = f"blk.{L}.{f}.weight"
            T[nm] = gen_norm(seed, 2 * tensor_id(nm), n)
    return T


# ----------------------------------------------------------------------------- hashes
_P1, _P2, _P3, _P4, _P5 = (0x9E3779B185EBCA87, 0xC2B2AE3D27D4EB4F, 0x165667B19E3779F9,
                           0x85EBCA77C2B2AE63, 0x27D4EB2F165667C5)


def _rotl(x, r):
    return ((x << r) | (x >> (64 - r))) & M64


def xxh64(data: bytes, seed: int = 0) -> int:
    """XXH64 (Yann Collet's published algorithm); the .sp-model table is sorted by it."""
    n = len(data)
    p = 0

    def rnd(acc, lane):
        acc = (acc + lane * _P2) & M64
        return (_rotl(acc, 31) * _P1) & M64

    def merge(acc, v):
        acc ^= rnd(0, v)
        return (acc * _P1 + _P4) & M64

    if n >= 32:
        v1 = (seed + _P1 + _P2) & M64
        v2 = (seed + _P2) & M64
        v3 = seed & M64
        v4 = (seed - _P1) & M64
        while p + 32 <= n:
            l1, l2, l3, l4 = struct.unpack_from("<4Q", data, p)
            v1, v2, v3, v4 = rnd(v1, l1), rnd(v2, l2), rnd(v3, l3), rnd(v4, l4)
            p += 32
        h = (_rotl(v1, 1) + _rotl(v2, 7) + _rotl(v3, 12) + _rotl(v4, 18)) & M64
        for v in (v1, v2, v3, v4):
            h = merge(h, v)
    else:
        h = (seed + _P5) & M64
    h = (h + n) & M64
    while p + 8 <= n:
        (k,) = struct.unpack_from("<Q", data, p)
        h ^= rnd(0, k)
        h = (_rotl(h, 27) * _P1 + _P4) & M64
        p += 8
    if p + 4 <= n:
        (k,) = struct.unpack_from("<I", data, p)
        h ^= (k * _P1) & M64
        h = (_rotl(h, 23) * _P2 + _P3) & M64
        p += 4
    while p < n:
        h ^= (data[p] * _P5) & M64
        h = (_rotl(h, 11) * _P1) & M64
        p += 1
    h ^= h >> 33
    h = (h * _P2) & M64
    h ^= h >> 29
    h = (h * _P3) & M64
    h ^= h >> 32
    return h


# ----------------------------------------------------------------------------- writer
DT_F32, DT_OK_Q4B, DT_BSCALE_F16 = 1, 13, 14
ARCH_WIRE = {ARCH_QWEN3: 2, ARCH_GEMMA3: 3}   # sp_model.h:60-69


def arch_info_bytes(cfg: Config) -> bytes:
    """The sp_arch_info prefix the loader memcpy's (sp_l1.h:78-97)."""
    b = struct.pack("<9If4B", ARCH_WIRE[cfg.arch], cfg.n_vocab, cfg.n_embd, cfg.n_layers,
                    cfg.n_head, cfg.n_head_kv, cfg.head_dim, cfg.max_context,
                    cfg.sliding_window, cfg.rope_base, 1 if cfg.gemma else 0,
                    1 if cfg.gemma else 0, 1 if cfg.gemma else 0, cfg.has_qk_norm)
    b += struct.pack("<IfI", cfg.n_ff, 1e-6, 1)
    return b


def write_sp_model(model_path: str, tok_path: str, cfg: Config, T: dict) -> None:
    """Write a `.sp-model` + paired `.sp-tokenizer` the reference loader accepts
    (magic/version/CRC-32/alignment/SHA-256 checks in sp_model_load.c:119-186)."""
    # tokenizer: header only (the forward path never reads the blob)
    th = bytearray(128)
    struct.pack_into("<IHHIIIIIIIQQ", th, 0, 0x4B545053, 0, 1, 128, 0, cfg.n_vocab,
                     0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 128, 0)
    struct.pack_into("<I", th, 52, zlib.crc32(bytes(th[:52])) & 0xFFFFFFFF)
    with open(tok_path, "wb") as f:
        f.write(th)
    tok_sha = hashlib.sha256(bytes(th)).digest()

    entries = []   # (name, dtype, dims, payload bytes-like)
    for name, t in T.items():
        if isinstance(t, Q4B):
            entries.append((name, DT_OK_Q4B, [t.cols, t.rows], t.codes))
            nblk = (t.cols + 31) // 32
            entries.append((name + ".bscale", DT_BSCALE_F16, [nblk, t.rows], t.bscale))
        else:
            entries.append((name, DT_F32, [t.size], np.ascontiguousarray(t, np.float32)))
    entries.sort(key=lambda e: xxh64(e[0].encode()))
    table_off = 512
    data_off = (table_off + 256 * len(entries) + 65535) // 65536 * 65536
    offs, cur = [], 0
    for e in entries:
        offs.append(cur)
        cur = (cur + e[3].nbytes + 63) // 64 * 64
    file_size = data_off + cur

    hdr = bytearray(512)
    ai = arch_info_bytes(cfg)
    struct.pack_into("<IHHIIII", hdr, 0, 0x444D5053, 0, 1, 512, ARCH_WIRE[cfg.arch], len(ai), 256)
    hdr[24:24 + len(ai)] = ai
    hdr[280:312] = tok_sha
    struct.pack_into("<IIQQQQQ", hdr, 312, cfg.n_vocab, len(entries), table_off, data_off,
                     file_size, 0, 0)
    struct.pack_into("<I", hdr, 360, zlib.crc32(bytes(hdr[:360])) & 0xFFFFFFFF)

    table = bytearray(256 * len(entries))
    for i, (name, dt, dims, arr) in enumerate(entries):
        o = 256 * i
        nm = name.encode()
        table[o:o + len(nm)] = nm
        esz = arr.itemsize
        struct.pack_into("<II8QQQII", table, o + 80, dt, len(dims), *(dims + [0] * (8 - len(dims))),
                         offs[i], arr.nbytes, esz, arr.nbytes // esz)
        struct.pack_into("<Q", table, o + 208, xxh64(nm))
    with open(model_path, "wb") as f:
        f.write(hdr)
        f.write(table)
        f.write(b"\0" * (data_off - 512 - len(table)))
        pos = 0
        for i, e in enumerate(entries):
            if offs[i] > pos:
                f.write(b"\0" * (offs[i] - pos))
                pos = offs[i]
            f.write(np.ascontiguousarray(e[3]).tobytes())
            pos += e[3].nbytes
        if cur > pos:
            f.write(b"\0" * (cur - pos))
