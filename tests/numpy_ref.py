"""An independent numpy restatement of the reference torso (`src/kernels.rs`, `src/engine.rs:463-522`),
used only to cross-check the C oracle on small inputs. It follows the WGSL's formulas and f16
rounding points but not its summation order, so comparisons with the oracle use a tolerance.
"""
import json
import os

import numpy as np

from strands_decider import model as M


def f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def silu(x):
    return x / (1.0 + np.exp(-x))


class NumpyTorso:
    def __init__(self, path):
        with open(os.path.join(path, "manifest.json")) as f:
            self.m = json.load(f)
        self.c = self.m["config"]
        self.shard = np.fromfile(os.path.join(path, "weights.0.bin"), np.uint8)
        e = self.m["embed"]
        rows = np.fromfile(os.path.join(path, e["rows"]), np.uint8)
        qb, sb = e["parts"][0][1], e["parts"][1][1]
        if e.get("u8"):
            rows = rows.reshape(e["vocab"], e["wire_row_bytes"])
            self.eq = rows[:, :qb]
            self.es = np.stack([M.decode_scales_u8(rows[r, qb:].tobytes(), 1, sb // 2)[0] for r in range(e["vocab"])])
        else:
            rows = rows.reshape(e["vocab"], e["row_bytes"])
            self.eq = rows[:, :qb]
            self.es = rows[:, qb:qb + sb].copy().view(np.float16)
        self.ebits = self.m["tensors"]["embed.q"]["bits"]
        self.cache = {}

    def raw(self, name):
        t = self.m["tensors"][name]
        return self.shard[t["offset"]:t["offset"] + t["bytes"]]

    def f32(self, name):
        return self.raw(name).view(np.float32)

    def w(self, name, f16_dequant):
        key = (name, f16_dequant)
        if key not in self.cache:
            t = self.m["tensors"][name + ".q"]
            n, k = t["N"], t["K"]
            q = self.raw(name + ".q").reshape(n, -1)
            s = self.raw(name + ".s").view(np.float16).reshape(n, -1)
            codes = M.unpack_codes(q, t["bits"], k).astype(np.float32) - float(1 << (t["bits"] - 1))
            sc = np.repeat(s.astype(np.float32), 32, axis=1)
            w = codes * sc
            self.cache[key] = f16(w) if f16_dequant else w
        return self.cache[key]

    def matmul(self, a, name):
        t = self.m["tensors"][name + ".q"]
        tiled = a.shape[0] > 20 and t["bits"] == 4 and t["group"] == 32 and not t.get("asym") and t["N"] % 64 == 0
        w = self.w(name, tiled)
        return f16(a.astype(np.float64) @ w.T.astype(np.float64))

    def forward(self, ids):
        """Full forward of one prompt from an empty state; returns the residual stream after each
        layer [n_layers][l][d] and the final-normed rows (all of them)."""
        c = self.c
        d, I = c["hidden_size"], c["intermediate_size"]
        H, DK, DV = c["linear_num_key_heads"], c["linear_key_head_dim"], c["linear_value_head_dim"]
        HQ, HK, HD, RD = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"], c["rotary_dim"]
        C = 2 * H * DK + H * DV
        l = len(ids)
        x = (M.unpack_codes(self.eq[ids], self.ebits, d).astype(np.float32) - float(1 << (self.ebits - 1))) \
            * np.repeat(self.es[ids].astype(np.float32), 32, axis=1)
        y = np.zeros((l, d), np.float32)

        def norm(x, w):
            return x / np.sqrt((x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True) + 1e-6) * w

        trace = []
        pos = np.arange(l)
        inv = c["rope_theta"] ** (-(2 * np.arange(RD // 2)) / RD)
        ang = pos[:, None] * inv[None, :]
        cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
        for i, kind in enumerate(c["layer_types"]):
            pre = f"layers.{i}."
            if i > 0:
                x = x + y
            h = f16(norm(x, self.f32(pre + "in_norm")))
            if kind == "adapter":
                y = f16(self.matmul(h, pre + "proj") + self.f32(pre + "bias"))
                trace.append(x + y)
                continue
            if kind == "linear_attention":
                big = self.matmul(h, pre + "in_proj")
                cw = self.f32(pre + "conv").reshape(C, 4)
                pad = np.concatenate([np.zeros((3, C), np.float32), big[:, :C]])
                s = sum(cw[:, j] * pad[j:j + l] for j in range(4))
                qkv = silu(s)
                q = qkv[:, :H * DK].reshape(l, H, DK)
                k = qkv[:, H * DK:2 * H * DK].reshape(l, H, DK)
                v = qkv[:, 2 * H * DK:].reshape(l, H, DV)
                a = big[:, C + H * DV:C + H * DV + H]
                b = big[:, C + H * DV + H:C + H * DV + 2 * H]
                beta = 1.0 / (1.0 + np.exp(-b))
                xx = a + self.f32(pre + "dt_bias")
                sp = np.where(xx > 20, xx, np.log1p(np.exp(np.minimum(xx, 20))))
                decay = np.exp(self.f32(pre + "neg_exp_A") * sp)
                S = np.zeros((H, DK, DV), np.float64)
                o = np.zeros((l, H, DV))
                for t in range(l):
                    qn = q[t] / np.sqrt((q[t] ** 2).sum(-1, keepdims=True) + 1e-6) / np.sqrt(DK)
                    kn = k[t] / np.sqrt((k[t] ** 2).sum(-1, keepdims=True) + 1e-6)
                    S = S * decay[t][:, None, None]
                    kv = np.einsum("hkv,hk->hv", S, kn)
                    delta = (v[t] - kv) * beta[t][:, None]
                    S = S + kn[:, :, None] * delta[:, None, :]
                    o[t] = np.einsum("hkv,hk->hv", S, qn)
                z = big[:, C:C + H * DV].reshape(l, H, DV)
                on = o / np.sqrt((o ** 2).mean(-1, keepdims=True) + 1e-6) * self.f32(pre + "gnorm") * silu(z)
                y = self.matmul(f16(on.reshape(l, H * DV)), pre + "out_proj")
            else:
                big = self.matmul(h, pre + "qkv")
                qh = big[:, :HQ * 2 * HD].reshape(l, HQ, 2, HD)
                qq, gate = qh[:, :, 0], qh[:, :, 1]
                kk = big[:, HQ * 2 * HD:HQ * 2 * HD + HK * HD].reshape(l, HK, HD)
                vv = big[:, HQ * 2 * HD + HK * HD:].reshape(l, HK, HD)

                def prep(t, w):
                    n = t / np.sqrt((t.astype(np.float64) ** 2).mean(-1, keepdims=True) + 1e-6) * w
                    r = n.copy()
                    r2 = RD // 2
                    c_, s_ = cos[:, None, :], sin[:, None, :]
                    r[..., :r2] = n[..., :r2] * c_ - n[..., r2:RD] * s_
                    r[..., r2:RD] = n[..., r2:RD] * c_ + n[..., :r2] * s_
                    return f16(r)
                Q = prep(qq, self.f32(pre + "q_norm"))
                K = prep(kk, self.f32(pre + "k_norm"))
                Q = f16(Q * (1.0 / np.sqrt(HD)))
                out = np.zeros((l, HQ, HD))
                mask = np.tril(np.ones((l, l), bool))
                for hh in range(HQ):
                    kh = hh // (HQ // HK)
                    sc = Q[:, hh].astype(np.float64) @ K[:, kh].T.astype(np.float64)
                    sc = np.where(mask, sc, -np.inf)
                    p = np.exp(sc - sc.max(-1, keepdims=True))
                    p /= p.sum(-1, keepdims=True)
                    out[:, hh] = (p @ vv[:, kh]) / (1.0 + np.exp(-gate[:, hh]))
                y = self.matmul(f16(out.reshape(l, HQ * HD)), pre + "o_proj")
            x = x + y
            h = f16(norm(x, self.f32(pre + "post_norm")))
            big = self.matmul(h, pre + "gate_up")
            mid = f16(silu(big[:, :I]) * big[:, I:])
            y = self.matmul(mid, pre + "down")
            trace.append(x + y)
        x = x + y
        return np.stack(trace), norm(x, self.f32("final_norm"))
