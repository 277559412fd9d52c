"""ctypes bindings for the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg to check the product; the product never imports it. See oracle.h for what it restates and its
parity status.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")


def build(force: bool = False) -> str:
    src = [os.path.join(HERE, f) for f in ("oracle.c", "oracle.h", "Makefile")]
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(os.path.getmtime(s) for s in src):
        subprocess.run(["make", "-C", HERE, "-s"], check=True)
    return LIB_PATH


class OrMat(C.Structure):
    _fields_ = [("q", C.c_void_p), ("s", C.c_void_p), ("b", C.c_void_p),
                ("n", C.c_int32), ("k", C.c_int32), ("bits", C.c_int32), ("group", C.c_int32), ("asym", C.c_int32)]


class OrLayer(C.Structure):
    _fields_ = [("kind", C.c_int32), ("in_norm", C.c_void_p), ("post_norm", C.c_void_p),
                ("in_proj", OrMat), ("out_proj", OrMat), ("conv", C.c_void_p), ("neg_a", C.c_void_p),
                ("dt_bias", C.c_void_p), ("gnorm", C.c_void_p), ("qkv", OrMat), ("o_proj", OrMat),
                ("q_norm", C.c_void_p), ("k_norm", C.c_void_p), ("proj", OrMat), ("bias", C.c_void_p),
                ("gate_up", OrMat), ("down", OrMat)]


class OrModel(C.Structure):
    _fields_ = [("d", C.c_int32), ("inter", C.c_int32), ("hq", C.c_int32), ("hk", C.c_int32), ("hd", C.c_int32),
                ("h", C.c_int32), ("dk", C.c_int32), ("dv", C.c_int32), ("rd", C.c_int32), ("vocab", C.c_int32),
                ("n_layers", C.c_int32), ("context", C.c_int32), ("rope_theta", C.c_double), ("embed", OrMat),
                ("final_norm", C.c_void_p), ("layers", C.POINTER(OrLayer))]


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(build())
        vp, i32 = C.c_void_p, C.c_int32
        _lib.or_engine_create.restype = vp
        _lib.or_engine_create.argtypes = [C.POINTER(OrModel)]
        _lib.or_engine_destroy.argtypes = [vp]
        _lib.or_forward.restype = C.c_int
        _lib.or_forward.argtypes = [vp, vp, i32, vp, i32, vp, i32, C.POINTER(vp), vp, vp]
        _lib.or_snapshot_len.restype = i32
        _lib.or_snapshot_len.argtypes = [vp]
        _lib.or_snapshot_free.argtypes = [vp]
        _lib.or_matmul.argtypes = [vp, i32, C.POINTER(OrMat), vp, i32]
        _lib.or_attn.argtypes = [vp, vp, vp, vp, i32, i32, i32, vp, i32, i32, i32, i32, i32, i32]
        _lib.or_gdn.argtypes = [vp, vp, i32, vp, i32, vp, vp, vp, i32, vp, i32, i32, i32, i32]
        _lib.or_head_probs.argtypes = [vp, i32, i32, vp, vp, vp, vp, vp, vp, i32, C.c_double, vp]
        _lib.or_decode_scales.argtypes = [vp, i32, i32, vp]
        _lib.or_f32_to_f16.restype = C.c_uint16
        _lib.or_f32_to_f16.argtypes = [C.c_float]
        _lib.or_f16_to_f32.restype = C.c_float
        _lib.or_f16_to_f32.argtypes = [C.c_uint16]
        _lib.or_set_threads.argtypes = [C.c_int]
        _lib.or_set_sum_reversed.argtypes = [C.c_int]
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def set_threads(n: int) -> None:
    lib().or_set_threads(n)


def set_sum_reversed(on: bool) -> None:
    """Perturbation probe: every matmul adds its f32 partial sums in the opposite order."""
    lib().or_set_sum_reversed(int(on))


def decode_scales(src: bytes, n: int, g: int) -> np.ndarray:
    buf = np.frombuffer(src, np.uint8).copy()
    out = np.empty((n, g), np.uint16)
    lib().or_decode_scales(_p(buf), n, g, _p(out))
    return out.view(np.float16)


def matmul(a: np.ndarray, q: np.ndarray, s: np.ndarray, n: int, k: int, bits: int = 4, group: int = 32,
           variant: int = 0, b: np.ndarray | None = None) -> np.ndarray:
    """Y = A W^T with the reference's dispatch for a.shape[0] rows (variant 0), or forced GEMV (1) /
    tiled (2). a: f16 [m, k]; b: the per-group f16 biases of an asymmetric weight."""
    a = np.ascontiguousarray(a, np.float16)
    q = np.ascontiguousarray(q)
    s = np.ascontiguousarray(s, np.float16)
    bb = None if b is None else np.ascontiguousarray(b, np.float16)
    w = OrMat(_p(q), _p(s), _p(bb) if bb is not None else None, n, k, bits, group, int(bb is not None))
    y = np.empty((a.shape[0], n), np.float16)
    lib().or_matmul(_p(a), a.shape[0], C.byref(w), _p(y), variant)
    return y


def attn(q, k, v, gate=None, gate_stride=0, gate_off=0, gate_step=0, p=0):
    """q [hq][l][hd], k/v [hk][lt][hd] f16 (rows p.. are this call's); gate [l][gate_stride]."""
    q = np.ascontiguousarray(q, np.float16)
    k = np.ascontiguousarray(k, np.float16)
    v = np.ascontiguousarray(v, np.float16)
    hq, l, hd = q.shape
    hk, lt, _ = k.shape
    out = np.empty((l, hq * hd), np.float16)
    g = None if gate is None else np.ascontiguousarray(gate, np.float16)
    lib().or_attn(_p(q), _p(k), _p(v), _p(g), gate_stride, gate_off, gate_step, _p(out), l, p, lt, hq, hk, hd)
    return out


def gdn(q, k, v, beta, decay, state=None):
    """One sequence. q/k [l][h][dk], v [l][h][dv] f32; beta/decay [l][h]. Returns (o [l][h*dv], state)."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    l, h, dk = q.shape
    dv = v.shape[2]
    beta = np.ascontiguousarray(beta, np.float32)
    decay = np.ascontiguousarray(decay, np.float32)
    st = np.zeros((h, dk, dv), np.float32) if state is None else np.array(state, np.float32, copy=True)
    o = np.empty((l, h * dv), np.float32)
    lib().or_gdn(_p(q), _p(k), h * dk, _p(v), h * dv, _p(beta), _p(decay), _p(st), int(state is not None), _p(o), l, h, dk, dv)
    return o, st


def head_probs(hidden: np.ndarray, head: dict, temperature: float) -> np.ndarray:
    hidden = np.ascontiguousarray(hidden, np.float32)
    nrows, d = hidden.shape
    t = {k: np.ascontiguousarray(v, np.float32) for k, v in head.items()}
    dim = t["q.weight"].shape[0]
    out = np.empty(nrows - 1, np.float64)
    lib().or_head_probs(_p(hidden), nrows, d, _p(t["norm.weight"]), _p(t["norm.bias"]), _p(t["q.weight"]),
                        _p(t["q.bias"]), _p(t["k.weight"]), _p(t["k.bias"]), dim, float(temperature), _p(out))
    return out


class Snapshot:
    def __init__(self, ptr):
        self.ptr = ptr

    @property
    def len(self) -> int:
        return lib().or_snapshot_len(self.ptr)

    def __del__(self):
        if self.ptr and _lib is not None:
            _lib.or_snapshot_free(self.ptr)
            self.ptr = None


KIND = {"linear_attention": 0, "full_attention": 1, "adapter": 2}


class Engine:
    """The oracle torso over a model directory in the reference's layout."""

    def __init__(self, model_dir: str):
        with open(os.path.join(model_dir, "manifest.json")) as f:
            m = json.load(f)
        self.manifest = m
        c = m["config"]
        self.d = c["hidden_size"]
        shard = np.memmap(os.path.join(model_dir, m["shards"][0]["path"]), dtype=np.uint8, mode="r")
        self._keep = [shard]
        tens = m["tensors"]

        def raw(name):
            t = tens[name]
            return shard[t["offset"]: t["offset"] + t["bytes"]]

        def f32(name):
            return raw(name).view(np.float32)

        def mat(name):
            t = tens[name + ".q"]
            qa = raw(name + ".q")
            sa = raw(name + ".s")
            ba = raw(name + ".b") if t.get("asym") else None
            return OrMat(_p(qa), _p(sa), _p(ba), t["N"], t["K"], t.get("bits", 4), t.get("group", 32), int(t.get("asym", False)))

        e = m["embed"]
        vocab = e["vocab"]
        data = np.fromfile(os.path.join(model_dir, e["rows"]), dtype=np.uint8)
        qb, sb = e["parts"][0][1], e["parts"][1][1]
        if e.get("u8"):
            rb = e["wire_row_bytes"]
            rows = data.reshape(vocab, rb)
            eq = np.ascontiguousarray(rows[:, :qb])
            es = np.empty((vocab, sb // 2), np.uint16)
            for r in range(vocab):
                es[r] = decode_scales(rows[r, qb:qb + 4 + sb // 2].tobytes(), 1, sb // 2).view(np.uint16)[0]
        else:
            rows = data.reshape(vocab, e["row_bytes"])
            eq = np.ascontiguousarray(rows[:, :qb])
            es = np.ascontiguousarray(rows[:, qb:qb + sb]).view(np.uint16)
        self._keep += [eq, es]
        et = tens["embed.q"]
        emb = OrMat(_p(eq), _p(es), None, vocab, c["hidden_size"], et.get("bits", 4), et.get("group", 32), int(et.get("asym", False)))

        layers = (OrLayer * len(c["layer_types"]))()
        for i, kind in enumerate(c["layer_types"]):
            pre = f"layers.{i}."
            L = layers[i]
            L.kind = KIND[kind]
            L.in_norm = _p(f32(pre + "in_norm"))
            if kind == "linear_attention":
                L.in_proj = mat(pre + "in_proj")
                L.out_proj = mat(pre + "out_proj")
                L.conv = _p(f32(pre + "conv"))
                L.neg_a = _p(f32(pre + "neg_exp_A"))
                L.dt_bias = _p(f32(pre + "dt_bias"))
                L.gnorm = _p(f32(pre + "gnorm"))
            elif kind == "full_attention":
                L.qkv = mat(pre + "qkv")
                L.o_proj = mat(pre + "o_proj")
                L.q_norm = _p(f32(pre + "q_norm"))
                L.k_norm = _p(f32(pre + "k_norm"))
            else:
                L.proj = mat(pre + "proj")
                L.bias = _p(f32(pre + "bias"))
            if kind != "adapter":
                L.post_norm = _p(f32(pre + "post_norm"))
                L.gate_up = mat(pre + "gate_up")
                L.down = mat(pre + "down")
        self._layers = layers
        self.model = OrModel(c["hidden_size"], c["intermediate_size"], c["num_attention_heads"], c["num_key_value_heads"],
                             c["head_dim"], c["linear_num_key_heads"], c["linear_key_head_dim"], c["linear_value_head_dim"],
                             c["rotary_dim"], vocab, len(c["layer_types"]), 4096, c["rope_theta"], emb,
                             _p(f32("final_norm")), layers)
        self.n_layers = len(c["layer_types"])
        self.ptr = lib().or_engine_create(C.byref(self.model))

    def forward(self, ids, rows, cache: Snapshot | None = None, keep: bool = False, trace: bool = False):
        """`Engine::forward`: returns (hidden [nrows][d] f32, snapshot or None, trace or None)."""
        ids = np.ascontiguousarray(ids, np.uint32)
        rows = np.ascontiguousarray(rows, np.int32)
        hidden = np.zeros((len(rows), self.d), np.float32)
        tr = np.zeros((self.n_layers, len(ids), self.d), np.float32) if trace else None
        snap = C.c_void_p()
        rc = lib().or_forward(self.ptr, _p(ids), len(ids), _p(rows), len(rows), cache.ptr if cache else None,
                              int(keep), C.byref(snap), _p(hidden), _p(tr))
        if rc != 0:
            raise ValueError(f"oracle forward failed ({rc})")
        return hidden, (Snapshot(snap.value) if keep else None), tr

    def __del__(self):
        if getattr(self, "ptr", None) and _lib is not None:
            _lib.or_engine_destroy(self.ptr)
            self.ptr = None
