"""fp32 torch-CPU restatement of the pi0.5 vision tower.  TEST INFRASTRUCTURE ONLY.

Written from the flax module the reference engine matched (openpi models/siglip.py:311-370, the
big_vision So400m/14 ViT, as docs/archive/windows/π05_네이티브엔진.md:29 cites it) and not from
pi05_oracle.cpp, so that the two restatements check each other:

  stem       nn.Conv(1152, 14x14, stride 14, VALID) on the [-1, 1] image, then + learned position
             embedding [256][1152] ("learn" posemb) -> x
  27 blocks  Encoder1DBlock (pre-LN):  y = LayerNorm(x); y = MultiHeadDotProductAttention(16 heads x 72,
             q/k/v/out Dense with bias)(y, y); x = x + y; y = LayerNorm(x); y = MlpBlock(x):
             Dense(4304) -> nn.gelu (tanh approximation, flax's default) -> Dense(1152); x = x + y
  encoder    LayerNorm "encoder_norm" (epsilon 1e-6, flax default)
  head       pool_type "none" keeps all 256 tokens per image; Dense(2048) "head" (num_classes = the
             Gemma width, openpi models/pi0.py:81-89)

Attention follows flax's dot_product_attention: the query is divided by sqrt(head_dim) cast to the
compute dtype (sqrt(72) = 8.485 -> bf16 8.5), logits = q k^T, softmax, weights . v.  With
`bf16=True` every module output is rounded to bf16 where the flax modules return the bf16 compute
dtype (dtype_mm = bfloat16): the conv input and output, the posemb sum, each LayerNorm, Dense and
residual sum, the scaled query, the logits, the softmax weights and the attention output; the
arithmetic inside each module is fp32.  Parameters come from the engine's seeded generator
(stream ids of behavior-2026_b200/csrc/pi05_model.h) and are bf16-valued.
"""
import numpy as np
import torch

import oracle as O

# generator stream ids (behavior-2026_b200/csrc/pi05_model.h)
(SIG_STEM_W, SIG_STEM_B, SIG_POSEMB, SIG_LN1_S, SIG_LN1_B, SIG_WQ, SIG_WK, SIG_WV, SIG_BQ, SIG_BK, SIG_BV, SIG_WO,
 SIG_BO, SIG_LN2_S, SIG_LN2_B, SIG_W1, SIG_B1, SIG_W2, SIG_B2, SIG_POST_S, SIG_POST_B, SIG_HEAD_W,
 SIG_HEAD_B) = range(1, 24)
W, MLP, HEADS, HD, PATCH, GEM_W = 1152, 4304, 16, 72, 14, 2048
GEM_EMBED = 30


def text_embedding(seed, tokens, bf16=True):
    """Gemma embedder (openpi models/gemma.py Embedder.encode): rows of the [257152][2048] table times
    sqrt(2048) cast to the table dtype (bf16 45.25 with bf16 tables), result in the compute dtype."""
    scale = float(torch.tensor(float(np.sqrt(2048.0))).to(torch.bfloat16)) if bf16 else float(np.sqrt(2048.0))
    rows = np.stack([O.gen_param_at(seed, GEM_EMBED, 0, int(t) * GEM_W, GEM_W) for t in tokens])
    e = torch.from_numpy(rows) * scale
    return (e.to(torch.bfloat16).float() if bf16 else e).numpy()


def prefix_embedding(seed, layers, images, tokens, bf16=True):
    """[image tokens of every camera ; text embeddings], [256 * n_cameras + n_text][2048]"""
    img = SiglipRef(layers, seed, bf16)(images)
    return np.concatenate([img, text_embedding(seed, tokens, bf16)], 0)


class SiglipRef:
    def __init__(self, layers, seed, bf16=True):
        self.layers, self.bf16 = layers, bf16
        p = lambda kind, sub, shape: torch.from_numpy(O.gen_param(seed, kind, sub, shape))
        # the generator lays the stem out as [out][(ky * 14 + kx) * 3 + channel]; flax's conv kernel is HWIO
        self.stem_w = p(SIG_STEM_W, 0, (W, PATCH, PATCH, 3)).permute(0, 3, 1, 2).contiguous()  # OIHW
        self.stem_b = p(SIG_STEM_B, 0, (W,))
        self.posemb = p(SIG_POSEMB, 0, (256, W))
        self.blocks = []
        for l in range(layers):
            self.blocks.append(dict(
                ln1_s=p(SIG_LN1_S, l, (W,)), ln1_b=p(SIG_LN1_B, l, (W,)),
                wq=p(SIG_WQ, l, (W, W)), wk=p(SIG_WK, l, (W, W)), wv=p(SIG_WV, l, (W, W)),
                bq=p(SIG_BQ, l, (W,)), bk=p(SIG_BK, l, (W,)), bv=p(SIG_BV, l, (W,)),
                wo=p(SIG_WO, l, (W, W)), bo=p(SIG_BO, l, (W,)),
                ln2_s=p(SIG_LN2_S, l, (W,)), ln2_b=p(SIG_LN2_B, l, (W,)),
                w1=p(SIG_W1, l, (MLP, W)), b1=p(SIG_B1, l, (MLP,)), w2=p(SIG_W2, l, (W, MLP)), b2=p(SIG_B2, l, (W,))))
        self.post_s = p(SIG_POST_S, 0, (W,))
        self.post_b = p(SIG_POST_B, 0, (W,))
        self.head_w = p(SIG_HEAD_W, 0, (GEM_W, W))
        self.head_b = p(SIG_HEAD_B, 0, (GEM_W,))

    def R(self, x):
        return x.to(torch.bfloat16).float() if self.bf16 else x

    def layernorm(self, x, s, b):
        mean = x.mean(-1, keepdim=True)
        var = ((x - mean) ** 2).mean(-1, keepdim=True)
        return self.R((x - mean) * torch.rsqrt(var + 1e-6) * s + b)

    def dense(self, x, w, b):
        return self.R(x @ w.t() + b)

    def attention(self, y, blk):
        n, T, _ = y.shape
        q = self.dense(y, blk["wq"], blk["bq"]).view(n, T, HEADS, HD)
        k = self.dense(y, blk["wk"], blk["bk"]).view(n, T, HEADS, HD)
        v = self.dense(y, blk["wv"], blk["bv"]).view(n, T, HEADS, HD)
        div = float(np.sqrt(np.float32(HD)))
        if self.bf16:
            div = float(torch.tensor(div).to(torch.bfloat16))
        q = self.R(q / div)
        logits = self.R(torch.einsum("nqhd,nkhd->nhqk", q, k))
        w = self.R(torch.softmax(logits, -1))
        o = self.R(torch.einsum("nhqk,nkhd->nqhd", w, v)).reshape(n, T, W)
        return self.dense(o, blk["wo"], blk["bo"])

    def __call__(self, images, points=None):
        """images uint8 [n_cameras][224][224][3] -> image tokens [n_cameras * 256][2048] (fp32 array).
        `points` (a dict) receives img.stem, img.l<N>.out, img.encoded."""
        img = torch.from_numpy(np.ascontiguousarray(images)).float().permute(0, 3, 1, 2)  # NCHW
        x = self.R(img / 127.5 - 1.0)
        x = self.R(torch.nn.functional.conv2d(x, self.stem_w, self.stem_b, stride=PATCH))  # [n][1152][16][16]
        n = x.shape[0]
        x = x.flatten(2).transpose(1, 2)  # [n][256][1152], row-major patches
        x = self.R(x + self.posemb[None])
        if points is not None:
            points["img.stem"] = x.reshape(-1).numpy().copy()
        for l, blk in enumerate(self.blocks):
            y = self.layernorm(x, blk["ln1_s"], blk["ln1_b"])
            x = self.R(x + self.attention(y, blk))
            y = self.layernorm(x, blk["ln2_s"], blk["ln2_b"])
            h = self.R(torch.nn.functional.gelu(self.dense(y, blk["w1"], blk["b1"]), approximate="tanh"))
            x = self.R(x + self.dense(h, blk["w2"], blk["b2"]))
            if points is not None:
                points[f"img.l{l}.out"] = x.reshape(-1).numpy().copy()
        x = self.layernorm(x, self.post_s, self.post_b)
        if points is not None:
            points["img.encoded"] = x.reshape(-1).numpy().copy()
        return self.dense(x, self.head_w, self.head_b).reshape(n * 256, GEM_W).numpy()
