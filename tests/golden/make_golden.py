"""Generate the golden vectors in this folder from the reference's own CPU oracles.

Run in a checkout that has the reference mounted (it imports it at run time; nothing is
copied):

    python tests/golden/make_golden.py --reference /path/to/supra2-img-web

Sources of truth:
  - DiT self / cross attention and the single-head VAE attention come from the reference's
    PyTorch oracle `attention()` (tools/reference.py:72-79), called exactly as its
    dit_forward calls it (tools/reference.py:96-100) with heads=9, and with heads=1 for the
    VAE shape (the app's VAE attention is ops.attention with H=1, D=512, app/models/vae.js:86).
  - The cross-attention ragged case is produced both per sequence at its true length (as the
    app runs it, app/models/dit.js:184) and padded+masked (as tools/reference.py:167-171 does).
  - T5 attention comes from Hugging Face transformers' T5Attention (the module
    tools/reference.py:129 runs): q/k/v projections with seeded weights, o = identity, and the
    relative-attention-bias embedding set to a seeded [32, 12] table; its compute_bias gives
    the [H, L, L] bias. transformers is not vendored by the reference (version recorded below).
  - Bucket vectors come from T5Attention._relative_position_bucket, which
    app/models/t5.js:13-23 restates.
  - The cross-attention K/V preparation (ctx_proj, then each block's cross_attn.kv) comes from
    the reference's `linear` (tools/reference.py:67-68), called as dit_forward calls it.

Output format is the reference's dump format (tools/reference.py:41-54): one raw
little-endian float32 file per tensor plus index.json with shapes and metadata.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


class Dump:
    def __init__(self, out):
        self.out = out
        self.index = {}

    def __call__(self, name, t, **meta):
        a = t.detach().float().contiguous().cpu().numpy() if torch.is_tensor(t) else np.asarray(t, dtype=np.float32)
        a.astype("<f4").tofile(os.path.join(self.out, name + ".bin"))
        self.index[name] = {"shape": list(a.shape), **meta}

    def save(self, **extra):
        with open(os.path.join(self.out, "index.json"), "w") as f:
            json.dump({**extra, "tensors": self.index}, f, indent=1, sort_keys=True)


def sha(t):
    return hashlib.sha256(t.detach().float().contiguous().numpy().astype("<f4").tobytes()).hexdigest()


@torch.no_grad()
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SUPRA_REFERENCE", ""))
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    if not args.reference:
        sys.exit("pass --reference <path to the reference checkout>")
    sys.path.insert(0, os.path.join(args.reference, "tools"))
    import reference  # tools/reference.py (imports only torch/numpy at module level)
    import transformers
    from transformers import T5Config
    from transformers.models.t5.modeling_t5 import T5Attention

    torch.set_num_threads(1)
    d = Dump(args.out)
    meta = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__,
            "transformers": transformers.__version__, "cases": {}}

    # ---- DiT self-attention, interleaved qkv [B, N, 1728] (app/models/dit.js:172) ----------
    for name, B, N, seed in (("dit_self", 2, 40, 11),):
        g = torch.Generator().manual_seed(seed)
        qkv = torch.randn(B, N, 3 * 576, generator=g)
        v3 = qkv.view(B, N, 3, 576)
        out = reference.attention(v3[:, :, 0], v3[:, :, 1], v3[:, :, 2], 9)
        d(f"{name}_qkv", qkv, seed=seed)
        d(f"{name}_out", out)
        meta["cases"][name] = {"B": B, "N": N, "H": 9, "D": 64, "seed": seed}

    # ---- config-1 size (B=2, 256 tokens): inputs regenerated from the seed, output stored ---
    g = torch.Generator().manual_seed(1)
    qkv = torch.randn(2, 256, 1728, generator=g)
    v3 = qkv.view(2, 256, 3, 576)
    out = reference.attention(v3[:, :, 0], v3[:, :, 1], v3[:, :, 2], 9)
    d("dit_self_cfg1_out", out, input_sha256=sha(qkv),
      inputs="torch.Generator().manual_seed(1); torch.randn(2, 256, 1728) as interleaved qkv")
    meta["cases"]["dit_self_cfg1"] = {"B": 2, "N": 256, "H": 9, "D": 64, "seed": 1}

    # ---- DiT cross-attention, ragged cached K/V [L, 1152] (app/models/dit.js:137-144,184) ---
    Ls = [1, 7, 77, 128]
    g = torch.Generator().manual_seed(22)
    B, N = len(Ls), 48
    q = torch.randn(B, N, 576, generator=g)
    kvs = [torch.randn(L, 1152, generator=g) for L in Ls]
    d("dit_cross_q", q, seed=22)
    per_seq = []
    for b, (L, kv) in enumerate(zip(Ls, kvs)):
        d(f"dit_cross_kv{b}", kv)
        o = reference.attention(q[b:b + 1], kv[None, :, :576], kv[None, :, 576:], 9)[0]
        per_seq.append(o)
    d("dit_cross_out", torch.stack(per_seq))
    # padded + masked form of the same batch (tools/reference.py:167-171)
    Lm = max(Ls)
    kp = torch.zeros(B, Lm, 576)
    vp = torch.zeros(B, Lm, 576)
    mask = torch.zeros(B, Lm)
    for b, (L, kv) in enumerate(zip(Ls, kvs)):
        kp[b, :L] = kv[:, :576]
        vp[b, :L] = kv[:, 576:]
        mask[b, :L] = 1
    d("dit_cross_out_masked", reference.attention(q, kp, vp, 9, mask))
    meta["cases"]["dit_cross"] = {"Ls": Ls, "N": N, "H": 9, "D": 64, "seed": 22}

    # ---- T5 encoder attention with relative-position bias (app/models/t5.js:73-80) ---------
    cfg = T5Config(d_model=768, d_kv=64, num_heads=12, relative_attention_num_buckets=32,
                   relative_attention_max_distance=128, dropout_rate=0.0, is_decoder=False)
    att = T5Attention(cfg, has_relative_attention_bias=True).eval()
    g = torch.Generator().manual_seed(33)
    for lin in (att.q, att.k, att.v):
        lin.weight.copy_(torch.randn(768, 768, generator=g) / 768 ** 0.5)
    att.o.weight.copy_(torch.eye(768))
    table = torch.randn(32, 12, generator=g) * 0.1
    att.relative_attention_bias.weight.copy_(table)
    d("t5_table", table, seed=33)
    t5_Ls = [1, 5, 37, 128]
    for L in t5_Ls:
        x = torch.randn(1, L, 768, generator=g)
        y = att(x)[0][0]
        d(f"t5_L{L}_q", att.q(x)[0])
        d(f"t5_L{L}_k", att.k(x)[0])
        d(f"t5_L{L}_v", att.v(x)[0])
        d(f"t5_L{L}_bias", att.compute_bias(L, L)[0])
        d(f"t5_L{L}_out", y)
    meta["cases"]["t5"] = {"Ls": t5_Ls, "H": 12, "D": 64, "scale": 1.0, "buckets": 32, "max_distance": 128}

    # ---- HF bucket function over a wide range of relative positions -------------------------
    rel = torch.arange(-1000, 1001)
    for nb, md in ((32, 128), (32, 64), (16, 32), (64, 256)):
        bk = T5Attention._relative_position_bucket(rel, bidirectional=True, num_buckets=nb, max_distance=md)
        d(f"bucket_{nb}_{md}", bk.float(), rel_first=-1000)
    meta["cases"]["buckets"] = {"rel": [-1000, 1000], "configs": [[32, 128], [32, 64], [16, 32], [64, 256]]}

    # ---- VAE mid-block single-head attention, D=512 (app/models/vae.js:77-94) ---------------
    g = torch.Generator().manual_seed(44)
    for name, T in (("vae_small", 96),):
        x = torch.randn(T, 512, generator=g)
        bound = (6.0 / 1024) ** 0.5
        W = [(torch.rand(512, 512, generator=g) * 2 - 1) * bound for _ in range(3)]
        bvec = [(torch.rand(512, generator=g) * 2 - 1) / 512 ** 0.5 for _ in range(3)]
        qv, kv_, vv = [x @ w.T + b for w, b in zip(W, bvec)]
        out = reference.attention(qv[None], kv_[None], vv[None], 1)[0]
        d(f"{name}_q", qv)
        d(f"{name}_k", kv_)
        d(f"{name}_v", vv)
        d(f"{name}_out", out)
        meta["cases"][name] = {"T": T, "H": 1, "D": 512, "seed": 44}

    # ---- cross-attention K/V preparation (app/models/dit.js:137-144): ctx_proj, then each block's
    # cross_attn.kv, through the reference's own `linear` (tools/reference.py:67-68) as its
    # dit_forward calls it (tools/reference.py:92,99); then one cross attention on block 1's K/V.
    # Inputs are regenerated from the seed in the order below (their SHA-256 is recorded).
    g = torch.Generator().manual_seed(55)
    L, nblk = 37, 3
    ctx = torch.randn(L, 768, generator=g)
    sd = {"ctx_proj.weight": torch.randn(576, 768, generator=g) / 768 ** 0.5,
          "ctx_proj.bias": torch.randn(576, generator=g) * 0.1}
    for i in range(nblk):
        sd[f"blocks.{i}.cross_attn.kv.weight"] = torch.randn(1152, 576, generator=g) / 576 ** 0.5
        sd[f"blocks.{i}.cross_attn.kv.bias"] = torch.randn(1152, generator=g) * 0.1
    qx = torch.randn(1, 48, 576, generator=g)
    p = reference.linear(sd, "ctx_proj", ctx)
    d("ctxprep_p", p, input_sha256=sha(torch.cat([ctx.reshape(-1)] + [t.reshape(-1) for t in sd.values()])))
    for i in range(nblk):
        d(f"ctxprep_kv{i}", reference.linear(sd, f"blocks.{i}.cross_attn.kv", p))
    kv1 = reference.linear(sd, "blocks.1.cross_attn.kv", p).view(1, L, 2, 576)
    d("ctxprep_cross_out", reference.attention(qx, kv1[:, :, 0], kv1[:, :, 1], 9)[0], q_sha256=sha(qx))
    meta["cases"]["ctxprep"] = {"L": L, "blocks": nblk, "seed": 55, "N": 48,
                                "inputs": "torch.Generator().manual_seed(55): ctx [37,768]; ctx_proj W [576,768]/sqrt(768), "
                                          "b [576]*0.1; per block kv W [1152,576]/sqrt(576), b [1152]*0.1; q [1,48,576]"}

    # ---- VAE mid-block attention (app/models/vae.js:77-94) as diffusers' attention block runs it:
    # GroupNorm(32, eps 1e-6) over the image, q/k/v linears, single-head attention (the
    # reference's own oracle, heads=1), output linear, residual add. torch's group_norm stands in
    # for diffusers (not installed); linears through the reference's `linear`. Inputs regenerated
    # from the seed in the order below (their SHA-256 recorded); only the output is stored.
    g = torch.Generator().manual_seed(66)
    hw, C = 64, 512
    x = torch.randn(hw, C, generator=g)
    vsd = {"norm.weight": 1.0 + 0.1 * torch.randn(C, generator=g), "norm.bias": 0.1 * torch.randn(C, generator=g)}
    for nm in ("q", "k", "v", "o"):
        vsd[nm + ".weight"] = torch.randn(C, C, generator=g) / C ** 0.5
        vsd[nm + ".bias"] = 0.1 * torch.randn(C, generator=g)
    n = F.group_norm(x.T[None], 32, vsd["norm.weight"], vsd["norm.bias"], eps=1e-6)[0].T
    qv, kv_, vv = (reference.linear(vsd, nm, n) for nm in ("q", "k", "v"))
    a = reference.attention(qv[None], kv_[None], vv[None], 1)[0]
    out = x + reference.linear(vsd, "o", a)
    d("vae_block_out", out, input_sha256=sha(torch.cat([x.reshape(-1)] + [t.reshape(-1) for t in vsd.values()])))
    meta["cases"]["vae_block"] = {"hw": hw, "C": C, "groups": 32, "eps": 1e-6, "seed": 66,
                                  "inputs": "torch.Generator().manual_seed(66): x [64,512]; norm weight 1+0.1*randn, "
                                            "bias 0.1*randn; q,k,v,o: W randn/sqrt(512), b 0.1*randn"}

    # ---- DiT block projections around the attention (app/models/dit.js:161-187) as dit_forward
    # runs them (tools/reference.py:96-100): self attention through the reference's oracle, the
    # gated output projection x + g1 * proj(a), then the ungated cross projection x + cproj(c).
    # mod is one step's modulation vector [6*576] shared by the batch (app/models/dit.js:164),
    # g1 = mod[2*576:3*576]. Inputs regenerated from the seed; only the outputs are stored.
    g = torch.Generator().manual_seed(99)
    B, N, D = 2, 64, 576
    x0 = torch.randn(B, N, D, generator=g)
    qkv = torch.randn(B, N, 3 * D, generator=g)
    mod = 0.5 * torch.randn(6 * D, generator=g)
    psd = {"proj.weight": torch.randn(D, D, generator=g) / D ** 0.5, "proj.bias": 0.1 * torch.randn(D, generator=g),
           "cproj.weight": torch.randn(D, D, generator=g) / D ** 0.5, "cproj.bias": 0.1 * torch.randn(D, generator=g)}
    cx = torch.randn(B, N, D, generator=g)
    v3 = qkv.view(B, N, 3, D)
    g1 = mod[2 * D:3 * D].expand(B, D)
    x1 = x0 + g1[:, None] * reference.linear(psd, "proj", reference.attention(v3[:, :, 0], v3[:, :, 1], v3[:, :, 2], 9))
    x2 = x1 + reference.linear(psd, "cproj", cx)
    ins = sha(torch.cat([x0.reshape(-1), qkv.reshape(-1), mod] + [t.reshape(-1) for t in psd.values()] + [cx.reshape(-1)]))
    d("dit_proj_x1", x1, input_sha256=ins)
    d("dit_proj_x2", x2)
    meta["cases"]["dit_proj"] = {"B": B, "N": N, "D": D, "seed": 99, "g_off": 2 * D,
                                 "inputs": "torch.Generator().manual_seed(99): x [2,64,576]; qkv [2,64,1728]; mod 0.5*randn "
                                           "[3456]; proj, cproj: W randn/sqrt(576), b 0.1*randn; c [2,64,576]"}

    # ---- one whole DiT block (app/models/dit.js:161-194) with the reference's own modulate,
    # layernorm, linear and attention, in dit_forward's order (tools/reference.py:96-102): the
    # step's modulation vector mod [6*576] stands for the adaLN linear's output (chunks shift,
    # scale, gate for the attention, then for the MLP), shared by the batch; the cross K/V of each
    # image is given (its prompt's prepared context, lengths 5 and 77). Only outputs stored.
    g = torch.Generator().manual_seed(111)
    B, N, D, Ls = 2, 64, 576, [5, 77]
    x0 = torch.randn(B, N, D, generator=g)
    mod = 0.5 * torch.randn(6 * D, generator=g)
    bsd = {}
    for nm, (o, i) in [("qkv", (3 * D, D)), ("proj", (D, D)), ("q", (D, D)), ("cproj", (D, D)),
                       ("fc1", (4 * D, D)), ("fc2", (D, 4 * D))]:
        bsd[nm + ".weight"] = torch.randn(o, i, generator=g) / i ** 0.5
        bsd[nm + ".bias"] = 0.1 * torch.randn(o, generator=g)
    kvs = [torch.randn(L, 2 * D, generator=g) for L in Ls]
    s1, c1, g1, s2, c2, g2 = (t.expand(B, D) for t in mod.view(6, D))
    qkv = reference.linear(bsd, "qkv", reference.modulate(reference.layernorm(x0), s1, c1)).view(B, -1, 3, D)
    x1 = x0 + g1[:, None] * reference.linear(bsd, "proj", reference.attention(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], 9))
    q = reference.linear(bsd, "q", reference.layernorm(x1))
    cx = torch.cat([reference.attention(q[b:b + 1], kvs[b][None, :, :D], kvs[b][None, :, D:], 9) for b in range(B)])
    x2 = x1 + reference.linear(bsd, "cproj", cx)
    mm = reference.linear(bsd, "fc2", F.gelu(reference.linear(bsd, "fc1", reference.modulate(reference.layernorm(x2), s2, c2)),
                                            approximate="tanh"))
    x3 = x2 + g2[:, None] * mm
    ins = sha(torch.cat([x0.reshape(-1), mod] + [t.reshape(-1) for t in bsd.values()] + [t.reshape(-1) for t in kvs]))
    d("dit_block_x1", x1, input_sha256=ins)
    d("dit_block_x2", x2)
    d("dit_block_x3", x3)
    meta["cases"]["dit_block"] = {"B": B, "N": N, "D": D, "Ls": Ls, "seed": 111,
                                  "inputs": "torch.Generator().manual_seed(111): x [2,64,576]; mod 0.5*randn [3456]; "
                                            "qkv, proj, q, cproj, fc1, fc2: W randn/sqrt(in), b 0.1*randn; kv [L,1152] "
                                            "per image"}

    d.save(**meta)
    print("wrote", args.out, len(d.index), "tensors")


if __name__ == "__main__":
    main()
