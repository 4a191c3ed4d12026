"""TEST INFRASTRUCTURE ONLY — a second, independent restatement of the reference's Gemma 3 forward
(crates/gem/src/model.rs:286-430) in numpy, used to cross-check the C++ oracle on small models.

Element-wise steps round in float32 exactly as the Rust code does; reductions are taken in float64
(the reference sums sequentially in float32), so agreement with the C++ oracle is to ~1e-5, not
bit-exact. Activation quantization uses round-half-to-even (the reference's SIMD paths)."""
from __future__ import annotations

import numpy as np

f32 = np.float32


def exp_fast(x):  # crates/nn/src/fast.rs:126-132
    x = np.asarray(x, f32)
    t = np.clip((x * f32(1.4426950408889634)).astype(f32), f32(-126), f32(126))
    n = np.floor((t + f32(0.5)).astype(f32)).astype(f32)
    f = (t - n).astype(f32)
    p = f32(1.540353039e-04)
    for c in (1.333355815e-03, 9.618129108e-03, 5.550410866e-02, 2.402265070e-01, 6.931471806e-01, 1.0):
        p = (f32(c) + (f * p).astype(f32)).astype(f32)
    return (p * np.ldexp(f32(1), n.astype(np.int32)).astype(f32)).astype(f32)


def tanh_fast(x):  # fast.rs:78-81
    e = exp_fast((f32(2) * np.clip(np.asarray(x, f32), f32(-10), f32(10))).astype(f32))
    return ((e - f32(1)).astype(f32) / (e + f32(1)).astype(f32)).astype(f32)


def rmsnorm(x, w, eps):  # model.rs:81-87
    ms = f32(np.sum(x.astype(np.float64) * x.astype(np.float64)) / len(x))
    r = f32(f32(1) / np.sqrt(f32(ms + f32(eps))))
    return ((x * r).astype(f32) * w).astype(f32)


def rmsnorm_inplace(x, w, eps):  # model.rs:89-95
    ms = f32(np.sum(x.astype(np.float64) * x.astype(np.float64)) / len(x))
    r = f32(f32(1) / np.sqrt(f32(ms + f32(eps))))
    return (x * (r * w).astype(f32)).astype(f32)


def quantize(x):  # q8.rs:207-222
    b = x.reshape(-1, 32)
    d = (np.abs(b).max(1) / f32(127)).astype(f32)
    inv = np.where(d > 0, f32(1) / np.where(d > 0, d, f32(1)), f32(0)).astype(f32)
    q = np.rint((b * inv[:, None]).astype(f32)).astype(np.int64)
    return q.reshape(-1), d


def matvec(W, s, x):
    """W: int8 [rows, cols] (or float weights with s None), s: [rows, cols/32] scales."""
    if s is None:
        return (W.astype(np.float64) @ x.astype(np.float64)).astype(f32)
    q, d = quantize(x)
    rows, cols = W.shape
    blk = (W.reshape(rows, cols // 32, 32).astype(np.int64) * q.reshape(1, cols // 32, 32)).sum(-1)
    scale = (s * d[None, :]).astype(f32).astype(np.float64)
    return (blk.astype(np.float64) * scale).sum(-1).astype(f32)


class Model:
    """Loads a gemma3 Q8_0 GGUF (gguf-py) and runs model.rs's forward for one sequence."""

    def __init__(self, path, ctx=256):
        import gguf
        r = gguf.GGUFReader(str(path))
        self.t = {t.name: t for t in r.tensors}
        f = {k: r.fields[k] for k in r.fields}

        def val(k):
            fld = f[k]
            return fld.parts[fld.data[0]][0]
        a = "gemma3"
        self.d = int(val(f"{a}.embedding_length"))
        self.nl = int(val(f"{a}.block_count"))
        self.nh = int(val(f"{a}.attention.head_count"))
        self.nkv = int(val(f"{a}.attention.head_count_kv"))
        self.hd = int(val(f"{a}.attention.key_length"))
        self.eps = f32(val(f"{a}.attention.layer_norm_rms_epsilon"))
        self.window = int(val(f"{a}.attention.sliding_window"))
        base = f32(val(f"{a}.rope.freq_base"))
        self.ctx = ctx
        half = self.hd // 2
        self.inv = [np.array([np.power(b, f32(-2.0) * f32(i) / f32(self.hd), dtype=f32) for i in range(half)], f32)
                    for b in (f32(10000), base)]
        self.kc = np.zeros((self.nl, ctx, self.nkv * self.hd), f32)
        self.vc = np.zeros((self.nl, ctx, self.nkv * self.hd), f32)

    def mat(self, name):
        t = self.t[name]
        rows, cols = int(t.shape[1]), int(t.shape[0])
        raw = np.ascontiguousarray(t.data).view(np.uint8).reshape(rows, cols // 32, 34)
        s = raw[:, :, :2].copy().view(np.float16).reshape(rows, cols // 32).astype(f32)
        q = raw[:, :, 2:].copy().view(np.int8).reshape(rows, cols)
        return q, s

    def vec(self, name):
        return np.array(self.t[name].data, f32).reshape(-1)

    def forward(self, tok, pos):
        d, hd, nh, nkv, eps = self.d, self.hd, self.nh, self.nkv, self.eps
        q, s = self.mat("token_embd.weight")
        x = ((q[tok].astype(f32) * np.repeat(s[tok], 32)).astype(f32) * np.sqrt(f32(d))).astype(f32)
        half = hd // 2
        rot = []
        for inv in self.inv:
            ang = (f32(pos) * inv).astype(f32)
            rot.append((np.sin(ang).astype(f32), np.cos(ang).astype(f32)))
        for l in range(self.nl):
            p = f"blk.{l}."
            swa = l % 6 < 5
            xn = rmsnorm(x, self.vec(p + "attn_norm.weight"), eps)
            qv = matvec(*self.mat(p + "attn_q.weight"), xn)
            kv = matvec(*self.mat(p + "attn_k.weight"), xn)
            vv = matvec(*self.mat(p + "attn_v.weight"), xn)
            sn, cs = rot[0 if swa else 1]
            qs = f32(f32(1) / np.sqrt(f32(hd)))

            def rope(v):
                a, b = v[:half].copy(), v[half:].copy()
                return np.concatenate([((a * cs).astype(f32) - (b * sn).astype(f32)).astype(f32),
                                       ((a * sn).astype(f32) + (b * cs).astype(f32)).astype(f32)])
            qn = self.vec(p + "attn_q_norm.weight")
            kn = self.vec(p + "attn_k_norm.weight")
            qh = [(rope(rmsnorm_inplace(qv[h * hd:(h + 1) * hd], qn, eps)) * qs).astype(f32) for h in range(nh)]
            kh = [rope(rmsnorm_inplace(kv[h * hd:(h + 1) * hd], kn, eps)) for h in range(nkv)]
            self.kc[l, pos] = np.concatenate(kh)
            self.vc[l, pos] = vv
            lo = max(0, pos + 1 - self.window) if swa else 0
            att = np.zeros(nh * hd, f32)
            G = nh // nkv
            for h in range(nh):
                g = h // G
                K = self.kc[l, lo:pos + 1, g * hd:(g + 1) * hd].astype(np.float64)
                V = self.vc[l, lo:pos + 1, g * hd:(g + 1) * hd].astype(np.float64)
                sc = (K @ qh[h].astype(np.float64)).astype(f32)
                e = exp_fast((sc - sc.max()).astype(f32))
                pr = (e * f32(f32(1) / f32(e.astype(np.float64).sum()))).astype(f32)
                att[h * hd:(h + 1) * hd] = (pr.astype(np.float64) @ V).astype(f32)
            o = matvec(*self.mat(p + "attn_output.weight"), att)
            o = rmsnorm_inplace(o, self.vec(p + "post_attention_norm.weight"), eps)
            x = (x + o).astype(f32)
            xn = rmsnorm(x, self.vec(p + "ffn_norm.weight"), eps)
            gt = matvec(*self.mat(p + "ffn_gate.weight"), xn)
            up = matvec(*self.mat(p + "ffn_up.weight"), xn)
            t = (f32(0.7978846) * (gt + (((f32(0.044715) * gt).astype(f32) * gt).astype(f32) * gt).astype(f32)).astype(f32)).astype(f32)
            t = tanh_fast(t)
            gg = ((((f32(0.5) * gt).astype(f32)) * (f32(1) + t).astype(f32)).astype(f32) * up).astype(f32)
            dn = matvec(*self.mat(p + "ffn_down.weight"), gg)
            dn = rmsnorm_inplace(dn, self.vec(p + "post_ffw_norm.weight"), eps)
            x = (x + dn).astype(f32)
        return rmsnorm(x, self.vec("output_norm.weight"), eps)
