"""Model directories in the reference's on-disk layout, and a seeded random-init writer for them.

A model directory holds (reference `src/model.rs:1-5`):

* ``manifest.json``: ``config`` (`src/model.rs:31-47`), ``shards`` (`:49-56`), ``tensors``
  (`:58-83`) and ``embed`` (`:92-103`);
* ``weights.<i>.bin``: each shard in GPU layout (`src/model.rs:110-112`);
* the embedding rows file (one row per token id, parts back to back, `src/model.rs:260-283`);
* ``tokenizer.json``, ``head.safetensors`` (`src/head.rs:25-52`) and ``hobson_config.json``
  (`src/lib.rs:90-98`).

Block-quantized matmul weights (`src/kernels.rs:6-13,545-586`): each weight row of K values is
stored as K/32 blocks. An int4 block is 4 u32 words, element e in word e/8 at bits 4(e%8), value
(q - 8) * scale. An int3 block is 3 u32 words: words 0 and 1 hold the low 2 bits of elements 0..15
and 16..31 at bits 2(e%16), word 2 holds the high bit of element e at bit e; value (q - 4) * scale.
An int2 block is 2 words like int3's first two; value (q - 2) * scale. Scales are fp16, one per
``group`` values; an asymmetric tensor has a per-group fp16 bias and value q * scale + bias.

There is no network here and no published checkpoint, so :func:`write_synthetic` draws the weights
from a seeded generator with the dims the reference's kernels are validated at
(`src/kernels.rs:813-835`): D=2048, I=6144, GDN 16 heads of 128x128, attention 8 query / 2 KV
heads of 256 with a 64-wide rotary part.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, field, asdict

import numpy as np

# Dims of the production model, from the reference's shape-validation test (`src/kernels.rs:813-835`)
# and the embedding size in its documentation (222 MB of int3 rows).
PROD = dict(
    hidden_size=2048,
    intermediate_size=6144,
    num_attention_heads=8,
    num_key_value_heads=2,
    head_dim=256,
    linear_num_key_heads=16,
    linear_key_head_dim=128,
    linear_value_head_dim=128,
    rms_norm_eps=1e-6,
    rope_theta=10_000_000.0,
    rotary_dim=64,
)
PROD_VOCAB = 248320
WRITER_VERSION = 2  # bumped whenever the seeded weights change
PROD_LAYERS = 24
HEAD_DIM_OUT = 256


def layer_pattern(n: int) -> list[str]:
    """Three gated-delta layers, then one full-attention layer, repeated (the builder's choice: the
    reference does not fix the pattern; it reads `layer_types` from the manifest)."""
    return ["full_attention" if i % 4 == 3 else "linear_attention" for i in range(n)]


@dataclass
class Config:
    hidden_size: int = 2048
    intermediate_size: int = 6144
    layer_types: list = field(default_factory=lambda: layer_pattern(PROD_LAYERS))
    num_attention_heads: int = 8
    num_key_value_heads: int = 2
    head_dim: int = 256
    linear_num_key_heads: int = 16
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10_000_000.0
    rotary_dim: int = 64
    unrotate: list | None = None

    @property
    def gdn_channels(self) -> int:
        """q, k, v channels of the fused in_proj output that go through the short conv."""
        h, dk, dv = self.linear_num_key_heads, self.linear_key_head_dim, self.linear_value_head_dim
        return 2 * h * dk + h * dv


def read_manifest(path: str) -> dict:
    """`model::read_manifest` (`src/model.rs:105-108`)."""
    with open(os.path.join(path, "manifest.json")) as f:
        return json.load(f)


# ---------------------------------------------------------------------------------------------
# Packing of quantized codes into the reference's GPU layout
# ---------------------------------------------------------------------------------------------

def pack_codes(q: np.ndarray, bits: int) -> np.ndarray:
    """Codes ``q`` (uint8, shape [N, K], K % 32 == 0) as the packed rows (uint8 [N, K*bits/8]) the
    reference's decoder reads (`src/kernels.rs:550-576`, `:63-89`)."""
    n, k = q.shape
    nb = k // 32
    qb = q.reshape(n, nb, 32).astype(np.uint32)
    if bits == 4:
        # byte j of a block = q[2j] | q[2j+1] << 4 (word e/8, nibble e%8, little-endian words)
        lo, hi = qb[:, :, 0::2], qb[:, :, 1::2]
        return (lo | (hi << 4)).astype(np.uint8).reshape(n, nb * 16)
    if bits in (2, 3):
        low = qb & 3
        sh = (2 * np.arange(16, dtype=np.uint32))[None, None, :]
        w0 = np.bitwise_or.reduce(low[:, :, :16] << sh, axis=2)
        w1 = np.bitwise_or.reduce(low[:, :, 16:] << sh, axis=2)
        words = [w0, w1]
        if bits == 3:
            hb = (qb >> 2) & 1
            w2 = np.bitwise_or.reduce(hb << np.arange(32, dtype=np.uint32)[None, None, :], axis=2)
            words.append(w2)
        w = np.stack(words, axis=2).astype("<u4")
        return w.view(np.uint8).reshape(n, nb * 4 * len(words))
    raise ValueError(f"unsupported bits {bits}")


def unpack_codes(packed: np.ndarray, bits: int, k: int) -> np.ndarray:
    """Inverse of :func:`pack_codes` (uint8 codes [N, K])."""
    n = packed.shape[0]
    nb = k // 32
    if bits == 4:
        b = packed.reshape(n, nb, 16)
        out = np.empty((n, nb, 32), np.uint8)
        out[:, :, 0::2] = b & 15
        out[:, :, 1::2] = b >> 4
        return out.reshape(n, k)
    nw = 3 if bits == 3 else 2
    w = packed.reshape(n, nb, nw * 4).copy().view("<u4").reshape(n, nb, nw).astype(np.uint32)
    sh = (2 * np.arange(16, dtype=np.uint32))[None, None, :]
    lo = np.concatenate([(w[:, :, 0:1] >> sh) & 3, (w[:, :, 1:2] >> sh) & 3], axis=2)
    if bits == 3:
        hi = (w[:, :, 2:3] >> np.arange(32, dtype=np.uint32)[None, None, :]) & 1
        lo = lo | (hi << 2)
    return lo.astype(np.uint8).reshape(n, k)


def dequant(packed: np.ndarray, scales: np.ndarray, bits: int, k: int, group: int = 32, bias=None) -> np.ndarray:
    """Weights as f32 [N, K]: (q - 2^(bits-1)) * scale, or q * scale + bias when asymmetric."""
    q = unpack_codes(packed, bits, k).astype(np.float32)
    s = np.repeat(scales.astype(np.float32).reshape(q.shape[0], -1), group, axis=1)
    if bias is not None:
        b = np.repeat(bias.astype(np.float32).reshape(q.shape[0], -1), group, axis=1)
        return q * s + b
    return (q - float(1 << (bits - 1))) * s


# ---------------------------------------------------------------------------------------------
# 8-bit log-scale codes (`src/model.rs:204-236`)
# ---------------------------------------------------------------------------------------------

def encode_scales_u8(scales: np.ndarray) -> tuple[bytes, np.ndarray]:
    """A per-row 8-bit code of fp16 scales [n, g]: a 4-byte header (m as fp16 bits, j as u16), then
    one code ``sign << 7 | k`` per scale, where |scale| ~ m 2^(-k j / 4096), m is the row's largest
    magnitude and the log step j spans the row's range in 127 codes. Returns the bytes and the fp16
    scales the codes decode to."""
    n, g = scales.shape
    s = scales.astype(np.float64)
    out = bytearray()
    heads = []
    codes = np.zeros((n, g), np.uint8)
    for r in range(n):
        mag = np.abs(s[r])
        m = float(np.float16(mag.max() or 1.0))
        lo = mag[mag > 0].min() if (mag > 0).any() else m
        j = int(min(65535, max(1, np.ceil(4096.0 * np.log2(m / lo) / 127.0))))
        heads.append(struct.pack("<eH", m, j))
        with np.errstate(divide="ignore"):
            kk = np.where(mag > 0, np.round(-np.log2(np.maximum(mag, 1e-30) / m) * 4096.0 / j), 127)
        kk = np.clip(kk, 0, 127).astype(np.uint8)
        codes[r] = kk | (np.signbit(s[r]).astype(np.uint8) << 7)
    for r in range(n):
        out += heads[r]
    out += codes.tobytes()
    return bytes(out), decode_scales_u8(bytes(out), n, g)


def decode_scales_u8(src: bytes, n: int, g: int) -> np.ndarray:
    """`decode_scales` (`src/model.rs:219-236`): |scale| = fp16(f32(m 2^(-k j / 4096))), computed
    in f64, rounded to f32, then to fp16 (round to nearest even); bit 7 of the code is the sign."""
    buf = np.frombuffer(src, np.uint8)
    head = buf[: 4 * n].view("<u2").reshape(n, 2)
    codes = buf[4 * n: 4 * n + n * g].reshape(n, g)
    out = np.empty((n, g), np.uint16)
    for r in range(n):
        m = float(head[r, 0:1].view(np.float16)[0])
        j = int(head[r, 1])
        k = (codes[r] & 127).astype(np.float64)
        mag = np.float16(np.float32(m * np.power(2.0, -(k * j) / 4096.0))).view(np.uint16)
        out[r] = mag | ((codes[r].astype(np.uint16) & 128) << 8)
    return out.view(np.float16)


# ---------------------------------------------------------------------------------------------
# Seeded random-init model
# ---------------------------------------------------------------------------------------------

def _code_lut(bits: int) -> np.ndarray:
    """A 256-entry table from a uniform byte to a code whose value (q - 2^(bits-1)) is a rounded,
    clipped Gaussian symmetric around 0 (so weight rows carry no systematic bias)."""
    half = 1 << (bits - 1)
    lim = half - 1
    u = (np.arange(256) + 0.5) / 256.0
    from math import erf, sqrt  # noqa: F401  (inverse CDF by bisection below)
    # inverse normal CDF by bisection, std chosen so the extreme codes are rare but present
    sd = lim / 2.5
    z = np.empty(256)
    for i, p in enumerate(u):
        lo, hi = -10.0, 10.0
        for _ in range(60):
            mid = 0.5 * (lo + hi)
            if 0.5 * (1.0 + erf(mid / sqrt(2.0))) < p:
                lo = mid
            else:
                hi = mid
        z[i] = 0.5 * (lo + hi)
    v = np.clip(np.round(z * sd), -lim, lim).astype(np.int32)
    return (v + half).astype(np.uint8)


_LUTS: dict[int, np.ndarray] = {}


def _codes(rng: np.random.Generator, n: int, k: int, bits: int) -> np.ndarray:
    if bits not in _LUTS:
        _LUTS[bits] = _code_lut(bits)
    return _LUTS[bits][rng.integers(0, 256, size=(n, k), dtype=np.uint8)]


def _quant_tensor(rng, n: int, k: int, bits: int, std: float, group: int = 32):
    """Packed codes and fp16 scales for an [n, k] weight whose values have roughly ``std``."""
    q = _codes(rng, n, k, bits)
    half = 1 << (bits - 1)
    qstd = float(np.std(_LUTS[bits].astype(np.float64) - half))
    jitter = rng.uniform(0.75, 1.25, size=(n, k // group)).astype(np.float32)
    scales = (std / qstd * jitter).astype(np.float16)
    return pack_codes(q, bits), scales


def _asym_bias(rng, scales: np.ndarray, bits: int) -> np.ndarray:
    """f16 biases for asymmetric codes: -2^(bits-1) scale (the symmetric centre) plus a per-group shift
    of up to half a scale."""
    s = scales.astype(np.float32)
    shift = rng.uniform(-0.5, 0.5, size=s.shape).astype(np.float32)
    return (-(float(1 << (bits - 1))) * s + shift * s).astype(np.float16)


class _ShardWriter:
    def __init__(self, path: str):
        self.f = open(path, "wb")
        self.off = 0
        self.tensors: dict[str, dict] = {}

    def add(self, name: str, data: np.ndarray, **meta):
        raw = np.ascontiguousarray(data).tobytes()
        pad = (-self.off) % 256  # every tensor starts 256-byte aligned
        if pad:
            self.f.write(b"\0" * pad)
            self.off += pad
        self.f.write(raw)
        t = {"offset": self.off, "bytes": len(raw), "shape": list(data.shape)}
        t.update(meta)
        self.tensors[name] = t
        self.off += len(raw)

    def add_matmul(self, rng, name: str, n: int, k: int, std: float, bits: int = 4, group: int = 32, asym: bool = False):
        packed, scales = _quant_tensor(rng, n, k, bits, std, group=group)
        self.add(f"{name}.q", packed, N=n, K=k, bits=bits, group=group, asym=asym)
        self.add(f"{name}.s", scales, N=n, K=k, bits=bits, group=group, asym=asym)
        if asym:  # value q * scale + bias: the symmetric values, each group shifted by up to half a scale
            self.add(f"{name}.b", _asym_bias(rng, scales, bits), N=n, K=k, bits=bits, group=group, asym=True)

    def close(self) -> int:
        self.f.close()
        return self.off


def write_synthetic(path: str, seed: int = 0, n_layers: int = PROD_LAYERS, vocab: int = PROD_VOCAB,
                    embed_bits: int = 3, embed_u8: bool = False, layer_types: list | None = None,
                    matmul_formats: list | None = None, dims: dict | None = None) -> dict:
    """Writes a complete model directory with seeded random-init weights in the reference's format.

    The dims are the production ones (:data:`PROD`), with ``dims`` overriding any of them (other
    sizes of the family); ``n_layers``/``vocab`` shrink test models. The
    init keeps the residual stream O(1): embedding rows of std 1, projections into the stream sized
    to add about 0.3 RMS each (from the typical RMS of their inputs), other projections
    1/sqrt(K). Returns the manifest."""
    os.makedirs(path, exist_ok=True)
    rng = np.random.default_rng(seed)
    types = layer_types or layer_pattern(n_layers)
    cfg = Config(layer_types=types, **{**PROD, **(dims or {})})
    d, i_size = cfg.hidden_size, cfg.intermediate_size
    h, dk, dv = cfg.linear_num_key_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim
    hq, hk, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    cc = cfg.gdn_channels
    in_n = -(-(cc + h * dv + 2 * h) // 64) * 64  # q,k,v | z | a | b, padded to 64 rows
    qkv_n = hq * hd * 2 + 2 * hk * hd
    add = 0.3  # RMS each residual projection adds

    def norm_w(n):
        return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    sw = _ShardWriter(os.path.join(path, "weights.0.bin"))
    if matmul_formats:  # (bits, group[, asym]) of the layer matmuls, in turn (the reference's other formats)
        fmts = iter(matmul_formats * 1000)
        plain_add = sw.add_matmul

        def add_fmt(rng_, name, n, k, std):
            f = next(fmts)  # (bits, group) or (bits, group, asym)
            plain_add(rng_, name, n, k, std, bits=f[0], group=f[1], asym=bool(f[2]) if len(f) > 2 else False)
        sw.add_matmul = add_fmt
    for li, kind in enumerate(types):
        pre = f"layers.{li}."
        sw.add(pre + "in_norm", norm_w(d))
        if kind == "linear_attention":
            sw.add_matmul(rng, pre + "in_proj", in_n, d, 1.0 / np.sqrt(d))
            sw.add(pre + "conv", (0.5 * rng.standard_normal((cc, 4))).astype(np.float32))
            a_log = rng.uniform(np.log(1.0), np.log(16.0), size=h)
            sw.add(pre + "neg_exp_A", (-np.exp(a_log)).astype(np.float32))
            dt = np.exp(rng.uniform(np.log(1e-3), np.log(0.1), size=h))
            sw.add(pre + "dt_bias", np.log(np.expm1(dt)).astype(np.float32))
            sw.add(pre + "gnorm", norm_w(dv))
            sw.add_matmul(rng, pre + "out_proj", d, h * dv, add / (np.sqrt(h * dv) * 0.6))
        elif kind == "full_attention":
            sw.add_matmul(rng, pre + "qkv", qkv_n, d, 1.0 / np.sqrt(d))
            sw.add(pre + "q_norm", norm_w(hd))
            sw.add(pre + "k_norm", norm_w(hd))
            sw.add_matmul(rng, pre + "o_proj", d, hq * hd, add / (np.sqrt(hq * hd) * 0.15))
        elif kind == "adapter":
            sw.add_matmul(rng, pre + "proj", d, d, add / np.sqrt(d))
            sw.add(pre + "bias", (0.01 * rng.standard_normal(d)).astype(np.float32))
            continue
        else:
            raise ValueError(kind)
        sw.add(pre + "post_norm", norm_w(d))
        sw.add_matmul(rng, pre + "gate_up", 2 * i_size, d, 1.0 / np.sqrt(d))
        sw.add_matmul(rng, pre + "down", d, i_size, add / (np.sqrt(i_size) * 0.5))
    sw.add("final_norm", norm_w(d))
    total = sw.close()
    tensors = sw.tensors

    # Embedding rows: [packed codes | fp16 scales] per token id (`src/model.rs:260-283`).
    nb = d // 32
    qbytes = nb * 4 * embed_bits
    sbytes = nb * 2
    erng = np.random.default_rng(seed + 1)
    rows_path = os.path.join(path, "embed.bin")
    wire_row = None
    with open(rows_path, "wb") as f:
        chunk = 16384
        for r0 in range(0, vocab, chunk):
            n = min(chunk, vocab - r0)
            packed, scales = _quant_tensor(erng, n, d, embed_bits, 1.0)
            if embed_u8:
                rows = []
                for r in range(n):
                    enc, _ = encode_scales_u8(scales[r:r + 1])
                    rows.append(packed[r].tobytes() + enc)
                f.write(b"".join(rows))
            else:
                f.write(np.concatenate([packed, scales.view(np.uint8).reshape(n, sbytes)], axis=1).tobytes())
    if embed_u8:
        wire_row = qbytes + 4 + nb
    tensors["embed.q"] = {"offset": 0, "bytes": 0, "shape": [vocab, qbytes], "N": vocab, "K": d,
                          "bits": embed_bits, "group": 32, "asym": False}
    embed = {"rows": "embed.bin", "vocab": vocab, "row_bytes": qbytes + sbytes,
             "parts": [["embed.q", qbytes], ["embed.s", sbytes]], "u8": bool(embed_u8)}
    if wire_row is not None:
        embed["wire_row_bytes"] = wire_row

    cfg_d = asdict(cfg)
    manifest = {"config": cfg_d, "shards": [{"path": "weights.0.bin", "start": 0, "bytes": total}],
                "tensors": tensors, "embed": embed, "tokenizer": "tokenizer.json",
                "synthetic": {"seed": seed, "n_layers": len(types), "vocab": vocab, "writer": WRITER_VERSION}}
    with open(os.path.join(path, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)

    # Pointer head: LayerNorm then q/k projections to HEAD_DIM_OUT (`src/head.rs:55-66`), sized so the
    # option logits (q.k / sqrt(dim)) have a standard deviation near 1.4: the spread of the reference's
    # example answer (0.874 / 0.065 / 0.062, logit gaps near 2.6, `README.md` of the reference).
    hrng = np.random.default_rng(seed + 2)
    head = {
        "norm.weight": (1.0 + 0.1 * hrng.standard_normal(d)).astype(np.float32),
        "norm.bias": (0.1 * hrng.standard_normal(d)).astype(np.float32),
        "q.weight": (hrng.standard_normal((HEAD_DIM_OUT, d)) / np.sqrt(d) * 1.2).astype(np.float32),
        "q.bias": (0.1 * hrng.standard_normal(HEAD_DIM_OUT)).astype(np.float32),
        "k.weight": (hrng.standard_normal((HEAD_DIM_OUT, d)) / np.sqrt(d) * 1.2).astype(np.float32),
        "k.bias": (0.1 * hrng.standard_normal(HEAD_DIM_OUT)).astype(np.float32),
    }
    write_safetensors(os.path.join(path, "head.safetensors"), head)
    with open(os.path.join(path, "hobson_config.json"), "w") as f:
        json.dump({"max_length": 4096, "temperature": 1.0,
                   "temperature_by_kind": {"noul": 1.0, "choice": 1.0, "score": 1.0},
                   "ordinal_smoothing": 0.0}, f)
    return manifest


def write_safetensors(path: str, tensors: dict[str, np.ndarray]) -> None:
    header = {}
    off = 0
    blobs = []
    for name, arr in tensors.items():
        raw = np.ascontiguousarray(arr, dtype=np.float32).tobytes()
        header[name] = {"dtype": "F32", "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hb = json.dumps(header).encode()
    hb += b" " * ((-len(hb)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


def read_safetensors(path: str) -> dict[str, np.ndarray]:
    with open(path, "rb") as f:
        data = f.read()
    n = struct.unpack("<Q", data[:8])[0]
    header = json.loads(data[8:8 + n])
    out = {}
    for name, e in header.items():
        if name == "__metadata__":
            continue
        a, b = e["data_offsets"]
        out[name] = np.frombuffer(data[8 + n + a: 8 + n + b], dtype=np.float32).reshape(e["shape"])
    return out


def ensure_model(path: str, **kw) -> str:
    """Writes the synthetic model at ``path`` unless a complete one with the same settings is there."""
    want = {"seed": kw.get("seed", 0), "n_layers": kw.get("n_layers", PROD_LAYERS), "vocab": kw.get("vocab", PROD_VOCAB),
            "writer": WRITER_VERSION}
    mpath = os.path.join(path, "manifest.json")
    if os.path.exists(mpath) and os.path.exists(os.path.join(path, "tokenizer.json")):
        try:
            m = read_manifest(path)
            if m.get("synthetic") == want and not kw.get("embed_u8") and not kw.get("layer_types"):
                return path
        except Exception:
            pass
    write_synthetic(path, **kw)
    from .tokenizer import write_synthetic_tokenizer
    write_synthetic_tokenizer(os.path.join(path, "tokenizer.json"), seed=kw.get("seed", 0))
    return path


# ---------------------------------------------------------------------------------------------
# The packed download format
# ---------------------------------------------------------------------------------------------

def write_packed(src: str, packed: str, unpacked: str) -> None:
    """From the GPU-layout model at ``src``, two directories holding the same weights.

    ``packed`` keeps its shard in the reference's packed download format, which `unpack_shard`
    (`src/model.rs:239-258`) converts:
    - tensors back to back, with a gap of 0-2 bytes after each (unaligned offsets);
    - every 2-D scale tensor (``*.s``) stored as 8-bit codes (``u8``);
    - the manifest's shard entry naming the packed file (``path``) and its size (``wire``);
    - no ``weights.0.bin``.

    ``unpacked`` is in GPU layout, with the scales the codes decode to: what the reference's
    download writes. The other files are symlinked to ``src``."""
    m = read_manifest(src)
    if len(m["shards"]) != 1:
        raise ValueError("one shard expected")
    with open(os.path.join(src, "weights.0.bin"), "rb") as f:
        data = bytearray(f.read())
    wire = bytearray()
    tensors = json.loads(json.dumps(m["tensors"]))
    order = sorted((t["offset"], name) for name, t in m["tensors"].items() if t.get("bytes", 0) > 0)
    for i, (off, name) in enumerate(order):
        t = tensors[name]
        raw = bytes(data[off:off + t["bytes"]])
        t["wire"] = len(wire)
        if name.endswith(".s") and len(t["shape"]) == 2:
            enc, dec = encode_scales_u8(np.frombuffer(raw, np.float16).reshape(t["shape"]))
            t["u8"] = True
            wire += enc
            data[off:off + t["bytes"]] = dec.tobytes()
        else:
            wire += raw
        wire += b"\x5a" * (i % 3)
    for out in (packed, unpacked):
        os.makedirs(out, exist_ok=True)
        for f in os.listdir(src):
            if f not in ("manifest.json", "weights.0.bin") and not os.path.exists(os.path.join(out, f)):
                os.symlink(os.path.abspath(os.path.join(src, f)), os.path.join(out, f))
    with open(os.path.join(packed, "weights.0.wire"), "wb") as f:
        f.write(wire)
    mp = json.loads(json.dumps(m))
    mp["tensors"] = tensors
    mp["shards"] = [{"path": "weights.0.wire", "start": 0, "bytes": m["shards"][0]["bytes"], "wire": len(wire)}]
    with open(os.path.join(packed, "manifest.json"), "w") as f:
        json.dump(mp, f)
    with open(os.path.join(unpacked, "weights.0.bin"), "wb") as f:
        f.write(data)
    with open(os.path.join(unpacked, "manifest.json"), "w") as f:
        json.dump(m, f)


def unpack_shard(wire: bytes, shard: dict, tensors: dict) -> bytes:
    """`unpack_shard` (`src/model.rs:239-258`) in numpy: each tensor with a ``wire`` offset in the
    shard's range goes to its offset, 8-bit scale codes decoded (`decode_scales`); the rest is zero."""
    out = bytearray(shard["bytes"])
    for name, t in tensors.items():
        w = t.get("wire")
        if w is None or not (shard["start"] <= t.get("offset", 0) < shard["start"] + shard["bytes"]):
            continue
        o = t["offset"] - shard["start"]
        if t.get("u8"):
            n, g = t["shape"]
            src = wire[w:w + 4 * n + n * g]
            if len(src) != 4 * n + n * g:
                raise ValueError(f"packed shard: {name} out of range")
            out[o:o + t["bytes"]] = decode_scales_u8(bytes(src), n, g).tobytes()
        else:
            src = wire[w:w + t["bytes"]]
            if len(src) != t["bytes"]:
                raise ValueError(f"packed shard: {name} out of range")
            out[o:o + t["bytes"]] = src
    return bytes(out)
