"""fp32 torch-CPU restatement of the pi0.5 LoRA training loss, with autograd gradients.  TEST INFRASTRUCTURE ONLY.

The forward is the openpi training loss the reference engine ported (docs/archive/windows/π05_네이티브엔진.md
:206-229; openpi models/pi0.py:189-214, models/lora.py): prefix (SigLIP image tokens + text embeddings)
and suffix (noisy actions) run jointly through the Gemma-2B / action-expert layers, the prefix attending
only to itself, the suffix to [prefix || suffix]; LoRA y = x W^T + (alpha/r) (x A^T) B^T with
alpha/r = 2 on q/k/v/o/gate/up/down of both stacks; loss = mean((v - u)^2).  Activations are rounded to
bf16 at the points the engine stores them (straight-through: rounding does not change gradients), all
arithmetic and every gradient is fp32.  Frozen weights come from the same seeded generator as the
engine and the C++ oracle; the prefix embedding comes from the C++ oracle (pi05_oracle.cpp).
"""
import math

import numpy as np
import torch

import oracle as O

# generator stream ids (behavior-2026_b200/csrc/pi05_model.h)
GEM_RMS1, GEM_WQ, GEM_WK, GEM_WV, GEM_WO, GEM_RMS2, GEM_WG, GEM_WU, GEM_WD = range(31, 40)
EXP_WQ, EXP_WK, EXP_WV, EXP_WO, EXP_WG, EXP_WU, EXP_WD = range(50, 57)
EXP_ADA1_W, EXP_ADA1_B, EXP_ADA2_W, EXP_ADA2_B, EXP_FINAL_W, EXP_FINAL_B = range(57, 63)
AIN_W, AIN_B, AOUT_W, AOUT_B, TIN_W, TIN_B, TOUT_W, TOUT_B = range(63, 71)
QD, HD = 2048, 256


def R(x):
    """round to bf16, gradient passes straight through"""
    return x + (x.to(torch.bfloat16).to(x.dtype) - x).detach()


def rope_table(npos):
    i = np.arange(128, dtype=np.float64)
    ts = np.power(10000.0, 2.0 * i / 256.0)
    a = np.arange(npos, dtype=np.float64)[:, None] / ts[None, :]
    return torch.from_numpy(np.cos(a).astype(np.float32)), torch.from_numpy(np.sin(a).astype(np.float32))


def time_embedding(t, w=1024):
    h = w // 2
    frac = np.arange(h, dtype=np.float64) / (h - 1)
    period = 4e-3 * np.power(4.0 / 4e-3, frac)
    a = float(t) * (2.0 * math.pi / period)
    return np.concatenate([np.sin(a), np.cos(a)]).astype(np.float32)


def lora_layout(L, gem_w=2048, exp_w=1024, gem_mlp=16384, exp_mlp=4096):
    """[(name, shape)] in the engine's flat order: stack, layer, (q,k,v), o, (gate, up), down; A then B."""
    out = []
    for s, (D, F) in enumerate(((gem_w, gem_mlp), (exp_w, exp_mlp))):
        for l in range(L):
            groups = [("q", D, QD), ("k", D, HD), ("v", D, HD), ("o", QD, D), ("g", D, F), ("u", D, F), ("d", F, D)]
            for name, K, Fa in groups:
                out.append((f"{'gem' if s == 0 else 'exp'}.{l}.{name}.A", (16, K)))
                out.append((f"{'gem' if s == 0 else 'exp'}.{l}.{name}.B", (Fa, 16)))
    return out


class LoraRef:
    def __init__(self, cfg, seed, flat_params, dtype=torch.float32):
        """dtype float64 gives a second computation of the same bf16-rounded network whose distance from
        the float32 one measures the floating-point floor of these comparisons"""
        torch.set_num_threads(max(1, torch.get_num_threads()))
        self.cfg = cfg
        self.seed = seed
        self.dtype = dtype
        self.L = cfg.gemma_layers
        P = lambda kind, sub, shape: torch.from_numpy(O.gen_param(seed, kind, sub, shape)).to(dtype)
        self.g, self.e = [], []
        for l in range(self.L):
            self.g.append(dict(rms1=P(GEM_RMS1, l, (2048,)), rms2=P(GEM_RMS2, l, (2048,)), q=P(GEM_WQ, l, (QD, 2048)),
                               k=P(GEM_WK, l, (HD, 2048)), v=P(GEM_WV, l, (HD, 2048)), o=P(GEM_WO, l, (2048, QD)),
                               g=P(GEM_WG, l, (16384, 2048)), u=P(GEM_WU, l, (16384, 2048)),
                               d=P(GEM_WD, l, (2048, 16384))))
            self.e.append(dict(q=P(EXP_WQ, l, (QD, 1024)), k=P(EXP_WK, l, (HD, 1024)), v=P(EXP_WV, l, (HD, 1024)),
                               o=P(EXP_WO, l, (1024, QD)), g=P(EXP_WG, l, (4096, 1024)), u=P(EXP_WU, l, (4096, 1024)),
                               d=P(EXP_WD, l, (1024, 4096))))
        NM = 2 * self.L + 1
        ws, bs = [], []
        for m in range(NM):
            fin = m == NM - 1
            kw = EXP_FINAL_W if fin else (EXP_ADA2_W if m & 1 else EXP_ADA1_W)
            l = 0 if fin else m // 2
            ws.append(P(kw, l, (3072, 1024)))
            bs.append(P(kw + 1, l, (3072,)))
        self.ada_w, self.ada_b = torch.stack(ws), torch.stack(bs)  # [NM][3072][1024], [NM][3072]
        self.ain_w, self.ain_b = P(AIN_W, 0, (1024, 32)), P(AIN_B, 0, (1024,))
        self.aout_w, self.aout_b = P(AOUT_W, 0, (32, 1024)), P(AOUT_B, 0, (32,))
        self.tin_w, self.tin_b = P(TIN_W, 0, (1024, 1024)), P(TIN_B, 0, (1024,))
        self.tout_w, self.tout_b = P(TOUT_W, 0, (1024, 1024)), P(TOUT_B, 0, (1024,))
        self.layout = lora_layout(self.L)
        self.params = {}
        off = 0
        flat = np.asarray(flat_params, np.float32)
        for name, shape in self.layout:
            n = shape[0] * shape[1]
            self.params[name] = torch.tensor(flat[off:off + n].reshape(shape), dtype=dtype, requires_grad=True)
            off += n
        assert off == flat.size, (off, flat.size)

    # ---- building blocks
    def lin(self, x, W, stack, l, name):
        A = R(self.params[f"{stack}.{l}.{name}.A"])
        B = R(self.params[f"{stack}.{l}.{name}.B"])
        U = 2.0 * R(x @ A.t())
        return R(x @ W.t() + U @ B.t())

    @staticmethod
    def rms(x, scale, shift=None):
        inv = 1.0 / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-6)
        y = x * inv * R(1.0 + scale)
        if shift is not None:
            y = y + shift
        return R(y)

    @staticmethod
    def rope(x, cos, sin):  # x [..., T, 256], cos/sin [T, 128]
        x1, x2 = x[..., :128], x[..., 128:]
        return R(torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1))

    @staticmethod
    def attend(q, k, v):  # q [nb,T,8,256], k/v [nb,S,256] -> [nb,T,2048]
        logits = torch.einsum("bthd,bsd->bhts", q, k)
        p = R(torch.softmax(logits, -1))
        o = torch.einsum("bhts,bsd->bthd", p, v)
        return R(o).reshape(q.shape[0], q.shape[1], QD)

    def qkv(self, x, W, stack, l, cos, sin):
        nb, T, _ = x.shape
        q = self.lin(x, W["q"], stack, l, "q").view(nb, T, 8, HD)
        k = self.lin(x, W["k"], stack, l, "k")
        v = self.lin(x, W["v"], stack, l, "v")
        q = self.rope(q, cos[:, None, :], sin[:, None, :]) * 0.0625
        k = self.rope(k, cos, sin)
        return q, k, v

    def mods(self, t):
        emb = torch.from_numpy(np.stack([time_embedding(tb) for tb in t])).to(self.dtype)
        c1 = emb @ self.tin_w.t() + self.tin_b
        c1 = c1 * torch.sigmoid(c1)
        c2 = c1 @ self.tout_w.t() + self.tout_b
        cond = R(c2 * torch.sigmoid(c2))
        m = torch.einsum("bk,mfk->bmf", cond, self.ada_w) + self.ada_b[None]
        return R(m).detach()  # [nb][NM][3072]

    # ---- the loss
    def loss(self, prefix_emb, actions, noise, t):
        a = torch.from_numpy(np.asarray(actions, np.float32)).to(self.dtype)
        eps = torch.from_numpy(np.asarray(noise, np.float32)).to(self.dtype)
        tt = torch.from_numpy(np.asarray(t, np.float32)).to(self.dtype)[:, None, None]
        xt = tt * eps + (1 - tt) * a
        u = eps - a
        v = self.velocity(prefix_emb, xt, t)
        return ((v - u) ** 2).mean()

    def velocity(self, prefix_emb, xt, t, points=None):
        """v = net(x_t, t, prefix) for a batch: prefix_emb [nb][P][2048], xt [nb][H][32] (tensor), t [nb].
        `points` (a dict) receives the prefix K/V cache of sample 0 per layer, pre.l<N>.k / .v."""
        nb, P, _ = prefix_emb.shape
        H = xt.shape[1]
        xp = torch.from_numpy(np.ascontiguousarray(prefix_emb, np.float32)).to(self.dtype)
        xs = R(xt.to(self.dtype) @ self.ain_w.t() + self.ain_b)
        md = self.mods(t)
        cos, sin = rope_table(P + H)
        cos, sin = cos.to(self.dtype), sin.to(self.dtype)
        cp, sp = cos[:P], sin[:P]
        cs, ss = cos[P:P + H], sin[P:P + H]
        for l in range(self.L):
            g, e = self.g[l], self.e[l]
            last = l == self.L - 1
            m1, m2 = md[:, 2 * l], md[:, 2 * l + 1]
            h1 = self.rms(xp, g["rms1"])
            qp, kp, vp = self.qkv(h1, g, "gem", l, cp, sp)
            if points is not None:
                points[f"pre.l{l}.k"] = kp[0].detach().double().numpy().ravel()
                points[f"pre.l{l}.v"] = vp[0].detach().double().numpy().ravel()
            h1s = self.rms(xs, m1[:, None, :1024], m1[:, None, 1024:2048])
            qs, ks, vs = self.qkv(h1s, e, "exp", l, cs, ss)
            os_ = self.attend(qs, torch.cat([kp, ks], 1), torch.cat([vp, vs], 1))
            if not last:
                op = self.attend(qp, kp, vp)
                xmid = R(xp + self.lin(op, g["o"], "gem", l, "o"))
                h2 = self.rms(xmid, g["rms2"])
                gg = self.lin(h2, g["g"], "gem", l, "g")
                uu = self.lin(h2, g["u"], "gem", l, "u")
                act = R(R(torch.nn.functional.gelu(gg, approximate="tanh")) * uu)
                xp = R(xmid + self.lin(act, g["d"], "gem", l, "d"))
            gate1, gate2 = m1[:, None, 2048:], m2[:, None, 2048:]
            xmid_s = R(xs + R(self.lin(os_, e["o"], "exp", l, "o") * gate1))
            h2s = self.rms(xmid_s, m2[:, None, :1024], m2[:, None, 1024:2048])
            gg = self.lin(h2s, e["g"], "exp", l, "g")
            uu = self.lin(h2s, e["u"], "exp", l, "u")
            act = R(R(torch.nn.functional.gelu(gg, approximate="tanh")) * uu)
            xs = R(xmid_s + R(self.lin(act, e["d"], "exp", l, "d") * gate2))
        mf = md[:, -1]
        hf = self.rms(xs, mf[:, None, :1024], mf[:, None, 1024:2048])
        return R(hf @ self.aout_w.t() + self.aout_b)

    def grads(self):
        out = []
        for n, shape in self.layout:
            g = self.params[n].grad
            out.append(np.zeros(shape[0] * shape[1], np.float32) if g is None else g.double().numpy().ravel())
        return np.concatenate(out)

    def named_slices(self):
        """{name: slice into the flat buffer}"""
        out, off = {}, 0
        for name, shape in self.layout:
            n = shape[0] * shape[1]
            out[name] = slice(off, off + n)
            off += n
        return out
