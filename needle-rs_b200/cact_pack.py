"""Writer for Needle 3 `.cact` v3 containers with seeded random-init weights.

The reference reads `.cact` v3 containers but ships no writer: upstream packs
them in `needle/model/export.py`, which is not vendored. This module writes the
layout the reference's reader parses, so synthetic models with the shipped
geometry can be built offline:

* header: 48 little-endian u32 words then `rope_theta` as f32
  (`crates/needle-infer/src/cact.rs:29-35, 344-390`);
* codebook: 28 f32, `cb2 | cb3 | cb4`, already scaled by `1/sqrt(group)`
  (`cact.rs:485-491`, `crates/needle-core/src/cq.rs:63-68`);
* directory: one 44-byte record per tensor, positional, no names
  (`cact.rs:398-425`);
* blobs: 64-byte aligned (`cact.rs:37-39`).

Tensors follow the canon `crates/needle-infer/src/v3.rs:236-332` walks:
embedding; per layer norm_in, q/k/v_proj, q/k/v_taps, q_norm, k_norm,
gate_proj, out_proj, post_norm, attn_gate, pre_hada, then the 13 HadamardMLP
tensors; the 9 mHC tensors; the two Hadamard permutations; 4 tensors per
Engram site; final_norm. Probe heads and the tokenizer record are optional
tails and are not written.

CQ packing follows the scheme documented at `crates/needle-core/src/cq.rs:4-19`:
per row and per group of 128, rotate by the normalised Walsh matrix, store the
group's L2 norm as FP16, and store the index of the codebook level nearest to
each coordinate of the unit vector, LSB-first in one continuous bitstream per
row (`cq.rs:908-925`). The quantisation rule itself (nearest level) is this
project's choice: the reference has no packer to pin it against.
"""
from __future__ import annotations

import dataclasses
import struct

import numpy as np

TAG_V3 = 0x05E12A84
HEADER_FMT = "<48If"
REC_FMT = "<BBHIIIIQQII"
REC_BYTES = 44
ALIGN = 64
DT_FP16, DT_FP32, DT_CQ, DT_RAW = 1, 2, 3, 4

# Lloyd-Max reconstruction levels for a unit Gaussian (Max 1960), positive
# halves; the negative half mirrors them.
_LLOYD_MAX = {
    2: (0.4528, 1.5104),
    3: (0.2451, 0.7560, 1.3439, 2.1520),
    4: (0.1284, 0.3881, 0.6568, 0.9424, 1.2562, 1.6181, 2.0690, 2.7326),
}


def f16_round(x) -> np.ndarray:
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def lloyd_codebook(group: int = 128) -> np.ndarray:
    """cb2|cb3|cb4 for coordinates of a unit vector in `group` dimensions,
    rounded through fp16 (every level is exactly representable in fp16)."""
    parts = []
    for bits in (2, 3, 4):
        half = np.array(_LLOYD_MAX[bits], np.float64)
        lv = np.concatenate([-half[::-1], half]) / np.sqrt(group)
        parts.append(lv)
    return f16_round(np.concatenate(parts))


def random_codebook(rng: np.random.Generator, std: float = 0.02) -> np.ndarray:
    """fp16-rounded N(0, std) codebook entries, as BASELINE config 0 draws them."""
    return f16_round(rng.normal(0.0, std, 28))


TERNARY = 5  # directory `bits` of a ternary tensor (cq.rs:55-61)
TERNARY_CENTROID = np.float32(1.2240064)
TERNARY_CRUMB = np.array([3, 0, 1], np.uint8)  # trit index 0, 1, 2 -> stored 2-bit crumb


def codebook_levels(codebook: np.ndarray, bits: int, group: int = 128) -> np.ndarray:
    """Levels of a width: slices cb2 | cb3 | cb4 of the header codebook, or the
    analytic ternary levels {-s, 0, +s}, s = centroid / sqrt(group) in f32."""
    if bits == TERNARY:
        s = TERNARY_CENTROID / np.sqrt(np.float32(group))
        return np.array([-s, 0.0, s], np.float32)
    start = {2: 0, 3: 4, 4: 12}[bits]
    return np.asarray(codebook[start:start + (1 << bits)], np.float32)


def walsh(n: int) -> np.ndarray:
    h = np.array([[1.0]], np.float64)
    while h.shape[0] < n:
        h = np.block([[h, h], [h, -h]])
    return h / np.sqrt(n)


def pack_indices(idx: np.ndarray, bits: int) -> np.ndarray:
    """LSB-first continuous bitstream per row: index k sits at bits
    [k*bits, (k+1)*bits) of its row (cq.rs:908-925)."""
    out, in_pad = idx.shape
    assert in_pad * bits % 8 == 0
    row_bytes = in_pad * bits // 8
    idx = idx.astype(np.uint64)
    if 8 % bits == 0:
        per = 8 // bits
        v = idx.reshape(out, row_bytes, per)
        byte = np.zeros((out, row_bytes), np.uint64)
        for j in range(per):
            byte |= v[:, :, j] << np.uint64(j * bits)
        return byte.astype(np.uint8)
    # 3 bits: eight indices fill three bytes.
    v = idx.reshape(out, in_pad // 8, 8)
    word = np.zeros((out, in_pad // 8), np.uint64)
    for j in range(8):
        word |= v[:, :, j] << np.uint64(j * bits)
    b = np.stack([(word >> np.uint64(8 * k)) & np.uint64(0xFF) for k in range(bits)], -1)
    return b.reshape(out, row_bytes).astype(np.uint8)


def unpack_indices(packed: np.ndarray, bits: int, in_pad: int) -> np.ndarray:
    out = packed.shape[0]
    bitpos = np.arange(in_pad, dtype=np.int64) * bits
    byte = bitpos // 8
    shift = bitpos % 8
    lo = packed[:, byte].astype(np.uint32)
    nxt = np.minimum(byte + 1, packed.shape[1] - 1)
    hi = np.where(shift + bits > 8, packed[:, nxt].astype(np.uint32), 0)
    return (((lo | (hi << 8)) >> shift.astype(np.uint32)) & ((1 << bits) - 1)).astype(np.uint8).reshape(out, in_pad)


def cq_blob(idx: np.ndarray, norms: np.ndarray, bits: int) -> bytes:
    """Packed indices followed by FP16 norms (cq.rs:181-238 reads this);
    ternary stores each trit index as its 2-bit crumb."""
    packed = pack_indices(TERNARY_CRUMB[idx], 2) if bits == TERNARY else pack_indices(idx, bits)
    return packed.tobytes() + np.asarray(norms, np.float32).astype("<f2").tobytes()


def cq_quantize(w: np.ndarray, bits: int, codebook: np.ndarray, group: int = 128,
                chunk_rows: int = 8192):
    """Quantise a dense [out, in] matrix. Returns (idx [out, in_pad] u8,
    norms [out, groups] f32 (fp16-exact))."""
    w = np.asarray(w, np.float32)
    out, in_feat = w.shape
    in_pad = -(-in_feat // group) * group
    ng = in_pad // group
    levels = codebook_levels(codebook, bits, group).astype(np.float64)
    order = np.argsort(levels, kind="stable")
    srt = levels[order]
    mids = (srt[1:] + srt[:-1]) / 2.0
    h = walsh(group)
    idx = np.empty((out, in_pad), np.uint8)
    norms = np.empty((out, ng), np.float32)
    for r0 in range(0, out, chunk_rows):
        r1 = min(out, r0 + chunk_rows)
        wp = np.zeros((r1 - r0, in_pad), np.float64)
        wp[:, :in_feat] = w[r0:r1]
        g = wp.reshape(r1 - r0, ng, group) @ h
        nrm = np.linalg.norm(g, axis=-1)
        nrm16 = f16_round(nrm)
        unit = g / np.where(nrm > 0, nrm, 1.0)[..., None]
        pos = np.searchsorted(mids, unit)
        idx[r0:r1] = order[pos].reshape(r1 - r0, in_pad).astype(np.uint8)
        norms[r0:r1] = nrm16
    return idx, norms


def random_cq(rng: np.random.Generator, out: int, in_feat: int, bits: int,
              group: int = 128, std: float = 0.02):
    """Indices uniform over the codebook and FP16 norms equal to ||H w_g|| of an
    N(0, std) draw — the kernel-benchmark inputs of BASELINE configs 0 and 1."""
    in_pad = -(-in_feat // group) * group
    ng = in_pad // group
    idx = rng.integers(0, 1 << bits, size=(out, in_pad), dtype=np.uint8)
    chi = np.sqrt(rng.chisquare(group, size=(out, ng))) * std
    return idx, f16_round(chi)


def dequantize(idx: np.ndarray, norms: np.ndarray, bits: int, codebook: np.ndarray,
               in_feat: int, group: int = 128) -> np.ndarray:
    """Dense reconstruction (cq.rs:763-779): levels*norm, then the rotation."""
    out, in_pad = idx.shape
    lv = codebook_levels(codebook, bits, group)[idx].reshape(out, in_pad // group, group)
    g = lv.astype(np.float64) * norms[..., None]
    return (g @ walsh(group)).reshape(out, in_pad)[:, :in_feat].astype(np.float32)


@dataclasses.dataclass
class Geometry:
    """Header geometry (cact.rs:306-390). Defaults are the shipped needle3
    geometry, as `tests/cact_v3_vectors.json` of the reference records it."""
    vocab_size: int = 8192
    out_vocab: int = 8192
    d_model: int = 768
    num_heads: int = 12
    num_kv_heads: int = 2
    num_layers: int = 20
    qk_head_dim: int = 48
    v_head_dim: int = 64
    max_seq_len: int = 8192
    hada_n: int = 1024
    mhc_lanes: int = 4
    sliding_window: int = 1024
    global_layers: tuple = (4, 9, 14, 19)
    qkv_conv_taps: int = 3
    engram_slots: int = 18432
    engram_sub_dim: int = 128
    engram_orders: tuple = (2, 3)
    engram_sites: tuple = (3, 7, 11, 15, 19)
    engram_conv_taps: int = 4
    engram_conv_dilation: int = 3
    engram_seed_heads: int = 0
    rope_theta: float = 100000.0
    kv_window: int = 256
    kv_bits: int = 8
    group: int = 128
    default_bits: int = 2
    embed_bits: int = 4
    mhc_bits: int = 4
    mlp_rank: int = 8

    @property
    def engram_heads(self) -> int:
        return self.d_model // (len(self.engram_orders) * self.engram_sub_dim)

    @property
    def num_tables(self) -> int:
        return len(self.engram_orders) * self.engram_heads

    def header_words(self, num_tensors: int) -> list:
        gmask = 0
        for l in self.global_layers:
            gmask |= 1 << l
        orders = list(self.engram_orders) + [0] * (4 - len(self.engram_orders))
        sites = list(self.engram_sites) + [0] * (16 - len(self.engram_sites))
        w = [TAG_V3, num_tensors, 28, self.kv_window, self.kv_bits, self.vocab_size,
             self.out_vocab, self.d_model, self.num_heads, self.num_kv_heads,
             self.num_layers, self.qk_head_dim, self.v_head_dim, self.max_seq_len,
             self.hada_n, self.mhc_lanes, self.sliding_window, gmask & 0xFFFFFFFF,
             gmask >> 32, self.qkv_conv_taps, self.engram_slots, self.engram_sub_dim,
             self.num_tables, self.engram_conv_taps, self.engram_conv_dilation,
             self.engram_seed_heads, len(self.engram_orders)] + orders + [len(self.engram_sites)] + sites
        assert len(w) == 48
        return w


def shipped() -> Geometry:
    return Geometry()


def tiny() -> Geometry:
    """A small geometry that keeps every structural feature of the shipped one:
    GQA, asymmetric head widths, local and global layers (with a window short
    enough to wrap), QKV conv, mHC lanes, two Engram sites and both CQ widths."""
    return Geometry(vocab_size=512, out_vocab=500, d_model=256, num_heads=4, num_kv_heads=2,
                    num_layers=4, qk_head_dim=16, v_head_dim=32, max_seq_len=96,
                    hada_n=256, mhc_lanes=4, sliding_window=8, global_layers=(1, 3),
                    qkv_conv_taps=3, engram_slots=64, engram_sub_dim=128,
                    engram_orders=(2, 3), engram_sites=(0, 2), engram_conv_taps=4,
                    engram_conv_dilation=3, rope_theta=10000.0)


class _Writer:
    def __init__(self):
        self.recs = []  # (dtype, shape, bytes, group, bits)

    def fp16(self, a):
        a = np.asarray(a, np.float32)
        self.recs.append((DT_FP16, a.shape, a.astype("<f2").tobytes(), 0, 0))

    def fp32(self, a):
        a = np.asarray(a, np.float32)
        self.recs.append((DT_FP32, a.shape, a.astype("<f4").tobytes(), 0, 0))

    def cq(self, shape, blob, group, bits):
        self.recs.append((DT_CQ, tuple(shape), blob, group, bits))

    def build(self, header_words, rope_theta, codebook) -> bytes:
        n = len(self.recs)
        head = struct.pack(HEADER_FMT, *header_words, np.float32(rope_theta))
        cb = np.asarray(codebook, "<f4").tobytes()
        dir_start = len(head) + len(cb)
        off = dir_start + n * REC_BYTES
        off = -(-off // ALIGN) * ALIGN
        dir_bytes = bytearray()
        body = bytearray()
        body_start = off
        for dtype, shape, blob, group, bits in self.recs:
            shp = list(shape) + [0] * (4 - len(shape))
            dir_bytes += struct.pack(REC_FMT, dtype, len(shape), 0, *shp, off, len(blob), group, bits)
            pad = off - (body_start + len(body))
            body += b"\0" * pad
            body += blob
            off = -(-(off + len(blob)) // ALIGN) * ALIGN
        pre = head + cb + bytes(dir_bytes)
        pre += b"\0" * (body_start - len(pre))
        return bytes(pre) + bytes(body)


def build_container(geom: Geometry | None = None, seed: int = 0,
                    codebook: np.ndarray | None = None, tokenizer: bytes | None = None,
                    confidence_head: bool = False) -> bytes:
    """A random-init Needle 3 container with `geom`'s geometry.

    Init profile (seeded, documented so parity runs are reproducible): CQ
    projections N(0, 0.02) quantised with the packer; Engram tables N(0, 0.5)
    and Engram key/value projections N(0, 0.05), so the Engram path moves the
    residual stream; norm scales and attention gates N(0, 0.02); QKV conv tap 0
    1+N(0, 0.1), later taps N(0, 0.3); HadamardMLP diagonals 1+N(0, 0.1), bias
    N(0, 0.1), Kronecker factors the normalised Walsh matrix plus N(0, 0.05),
    conditioning N(0, 0.1); mHC a_* 1+N(0, 0.1), b_* N(0, 0.1); Engram taps
    N(0, 0.5); permutations uniformly random.
    """
    g = geom or shipped()
    rng = np.random.default_rng(seed)
    cb = lloyd_codebook(g.group) if codebook is None else np.asarray(codebook, np.float32)
    d, L, n = g.d_model, g.num_layers, g.mhc_lanes
    qd, kd, vd = g.num_heads * g.qk_head_dim, g.num_kv_heads * g.qk_head_dim, g.num_kv_heads * g.v_head_dim
    od = g.num_heads * g.v_head_dim
    hn = g.hada_n
    bits_log2 = (hn - 1).bit_length()
    ba = 1 << (bits_log2 // 2)
    bb = hn // ba
    w = _Writer()

    def cqw(out, inp, bits, std):
        m = rng.normal(0.0, std, (out, inp)).astype(np.float32)
        idx, nrm = cq_quantize(m, bits, cb, g.group)
        w.cq((out, inp), cq_blob(idx, nrm, bits), g.group, bits)

    cqw(g.vocab_size, d, g.embed_bits, 0.02)
    for _ in range(L):
        w.fp16(rng.normal(0, 0.02, d))  # norm_in
        cqw(qd, d, g.default_bits, 0.02)
        cqw(kd, d, g.default_bits, 0.02)
        cqw(vd, d, g.default_bits, 0.02)
        if g.qkv_conv_taps:
            for dim in (qd, kd, vd):
                taps = rng.normal(0, 0.3, (g.qkv_conv_taps, dim))
                taps[0] = 1.0 + rng.normal(0, 0.1, dim)
                w.fp16(taps)
        w.fp16(rng.normal(0, 0.02, g.qk_head_dim))  # q_norm
        w.fp16(rng.normal(0, 0.02, g.qk_head_dim))  # k_norm
        cqw(od, d, g.default_bits, 0.02)  # gate_proj
        cqw(d, od, g.default_bits, 0.02)  # out_proj
        w.fp16(rng.normal(0, 0.02, d))  # post_norm
        w.fp16(rng.normal(0, 0.02, 1))  # attn_gate
        w.fp16(rng.normal(0, 0.02, d))  # pre_hada
        for _k in range(2):  # d1, d2
            w.fp16(1.0 + rng.normal(0, 0.1, hn))
        w.fp16(rng.normal(0, 0.1, hn))  # b2
        for _k in range(2):  # d3, d4
            w.fp16(1.0 + rng.normal(0, 0.1, hn))
        for _k in range(3):  # (w1a, w1b), (w2a, w2b), (w3a, w3b)
            w.fp16(walsh(ba) + rng.normal(0, 0.05, (ba, ba)))
            w.fp16(walsh(bb) + rng.normal(0, 0.05, (bb, bb)))
        w.fp16(rng.normal(0, 0.1, (d, g.mlp_rank)))  # cond_v
        w.fp16(rng.normal(0, 0.1, (g.mlp_rank, hn)))  # cond_u
    for _k in range(3):  # a_pre, a_post, a_res
        w.fp16(1.0 + rng.normal(0, 0.1, L))
    w.fp16(rng.normal(0, 0.1, (L, n)))  # b_pre
    w.fp16(rng.normal(0, 0.1, (L, n)))  # b_post
    w.fp16(rng.normal(0, 0.1, (L, n, n)))  # b_res
    cqw(L * n, n * d, g.mhc_bits, 0.02)  # phi_pre
    cqw(L * n, n * d, g.mhc_bits, 0.02)  # phi_post
    cqw(L * n * n, n * d, g.mhc_bits, 0.02)  # phi_res
    w.fp32(rng.permutation(hn).astype(np.float32))  # hada p1
    w.fp32(rng.permutation(hn).astype(np.float32))  # hada p2
    for _s in g.engram_sites:
        cqw(g.num_tables * g.engram_slots, g.engram_sub_dim, g.default_bits, 0.5)
        cqw(d, d, g.default_bits, 0.05)  # key_proj
        cqw(d, d, g.default_bits, 0.05)  # value_proj
        w.fp16(rng.normal(0, 0.5, (g.engram_conv_taps, d)))  # taps
    w.fp16(rng.normal(0, 0.02, d))  # final_norm
    if confidence_head:
        # heads.manifest [2] (confidence), then the head in canon order
        # (v3.rs:491-560): probes [(L+1)*4, d] CQ, gain [L+1, 4], query [4, d]
        # CQ, row_bias [4, L+1, 4], proj [1, 4*d] CQ, bias [1].
        kp, qn = 4, 4
        w.fp16(np.array([2.0]))
        cqw((L + 1) * kp, d, g.mhc_bits, 0.05)
        w.fp16(1.0 + rng.normal(0, 0.1, (L + 1, kp)))
        cqw(qn, d, g.mhc_bits, 0.05)
        w.fp16(rng.normal(0, 0.1, (qn, L + 1, kp)))
        cqw(1, qn * d, g.mhc_bits, 0.05)
        w.fp16(rng.normal(0, 0.1, 1))
    if tokenizer is not None:  # the RAW tokenizer record, last as in the shipped container
        w.recs.append((DT_RAW, (), bytes(tokenizer), 0, 0))
    return w.build(g.header_words(len(w.recs)), g.rope_theta, cb)


def read_directory(raw: bytes):
    """Parse header words, codebook and directory (for tests and tools)."""
    words = struct.unpack_from(HEADER_FMT, raw, 0)
    n = words[1]
    cb = np.frombuffer(raw, "<f4", 28, 49 * 4).copy()
    recs = []
    off = 49 * 4 + 28 * 4
    for i in range(n):
        dtype, ndim, _pad, s0, s1, s2, s3, o, nb, grp, bits = struct.unpack_from(REC_FMT, raw, off + i * REC_BYTES)
        recs.append(dict(index=i, dtype=dtype, ndim=ndim, shape=[s0, s1, s2, s3][:ndim],
                         offset=o, nbytes=nb, group=grp, bits=bits))
    return words, cb, recs
