import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "supra2-img-web_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run on the GPU box")


class Golden:
    """The golden vectors in tests/golden (reference dump format, tools/reference.py:41-54)."""

    def __init__(self, root=GOLDEN):
        self.root = root
        with open(os.path.join(root, "index.json")) as f:
            self.index = json.load(f)

    def __call__(self, name):
        meta = self.index["tensors"][name]
        a = np.fromfile(os.path.join(self.root, name + ".bin"), dtype="<f4")
        return a.reshape(meta["shape"])

    def meta(self, name):
        return self.index["tensors"][name]

    @property
    def cases(self):
        return self.index["cases"]


@pytest.fixture(scope="session")
def golden():
    return Golden()


def ctxprep_inputs():
    """Inputs of the golden 'ctxprep' case (cross-attention K/V preparation), regenerated from
    its seed in tests/golden/make_golden.py's order: ctx, ctx_proj weight and bias, then each
    block's kv weight and bias, then the cross-attention query."""
    import torch

    g = torch.Generator().manual_seed(55)
    L, nblk = 37, 3
    ctx = torch.randn(L, 768, generator=g)
    wp = torch.randn(576, 768, generator=g) / 768 ** 0.5
    bp = torch.randn(576, generator=g) * 0.1
    wkv, bkv = [], []
    for _ in range(nblk):
        wkv.append(torch.randn(1152, 576, generator=g) / 576 ** 0.5)
        bkv.append(torch.randn(1152, generator=g) * 0.1)
    qx = torch.randn(1, 48, 576, generator=g)
    flat = torch.cat([ctx.reshape(-1), wp.reshape(-1), bp.reshape(-1)] +
                     [t.reshape(-1) for pair in zip(wkv, bkv) for t in pair])
    return {"L": L, "ctx": ctx.numpy(), "wp": wp.numpy(), "bp": bp.numpy(), "wkv": [w.numpy() for w in wkv],
            "bkv": [b.numpy() for b in bkv], "q": qx[0].numpy(), "flat": flat.numpy(), "q_flat": qx.reshape(-1).numpy()}


def dit_proj_inputs():
    """Inputs of the golden 'dit_proj' case (the DiT block's projections around its attention),
    regenerated from its seed in tests/golden/make_golden.py's order."""
    import torch

    g = torch.Generator().manual_seed(99)
    B, N, D = 2, 64, 576
    x0 = torch.randn(B, N, D, generator=g)
    qkv = torch.randn(B, N, 3 * D, generator=g)
    mod = 0.5 * torch.randn(6 * D, generator=g)
    t = [torch.randn(D, D, generator=g) / D ** 0.5, 0.1 * torch.randn(D, generator=g),
         torch.randn(D, D, generator=g) / D ** 0.5, 0.1 * torch.randn(D, generator=g)]
    cx = torch.randn(B, N, D, generator=g)
    flat = torch.cat([x0.reshape(-1), qkv.reshape(-1), mod] + [u.reshape(-1) for u in t] + [cx.reshape(-1)])
    return {"B": B, "N": N, "D": D, "x0": x0.numpy(), "qkv": qkv.numpy(), "mod": mod.numpy(), "wp": t[0].numpy(),
            "bp": t[1].numpy(), "wc": t[2].numpy(), "bc": t[3].numpy(), "c": cx.numpy(), "flat": flat.numpy()}


def dit_block_inputs():
    """Inputs of the golden 'dit_block' case (one whole DiT block), regenerated from its seed in
    tests/golden/make_golden.py's order."""
    import torch

    g = torch.Generator().manual_seed(111)
    B, N, D, Ls = 2, 64, 576, [5, 77]
    x0 = torch.randn(B, N, D, generator=g)
    mod = 0.5 * torch.randn(6 * D, generator=g)
    w = {}
    for nm, (o, i) in [("qkv", (3 * D, D)), ("proj", (D, D)), ("q", (D, D)), ("cproj", (D, D)),
                       ("fc1", (4 * D, D)), ("fc2", (D, 4 * D))]:
        w[nm] = torch.randn(o, i, generator=g) / i ** 0.5
        w["b" + nm] = 0.1 * torch.randn(o, generator=g)
    kvs = [torch.randn(L, 2 * D, generator=g) for L in Ls]
    flat = torch.cat([x0.reshape(-1), mod] + [t.reshape(-1) for t in w.values()] + [t.reshape(-1) for t in kvs])
    return {"B": B, "N": N, "D": D, "Ls": Ls, "x0": x0.numpy(), "mod": mod.numpy(),
            "w": {k: v.numpy() for k, v in w.items()}, "kv": [t.numpy() for t in kvs], "flat": flat.numpy()}


@pytest.fixture(scope="session")
def gpu():
    """One libsupra_attn context on cuda:0, running on torch's current stream."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import supra_attn

    g = supra_attn.GPU(0, stream=torch.cuda.current_stream())
    yield g
    g.close()


def vae_block_inputs():
    """Inputs of the golden 'vae_block' case (VAE mid-block attention), regenerated from its seed
    in tests/golden/make_golden.py's order: x, the norm's weight and bias, then q, k, v, o weights
    and biases."""
    import torch

    g = torch.Generator().manual_seed(66)
    hw, C = 64, 512
    x = torch.randn(hw, C, generator=g)
    sd = {"gamma": 1.0 + 0.1 * torch.randn(C, generator=g), "beta": 0.1 * torch.randn(C, generator=g)}
    for nm in ("q", "k", "v", "o"):
        sd["w" + nm] = torch.randn(C, C, generator=g) / C ** 0.5
        sd["b" + nm] = 0.1 * torch.randn(C, generator=g)
    flat = torch.cat([x.reshape(-1)] + [t.reshape(-1) for t in sd.values()])
    return {"hw": hw, "C": C, "x": x.numpy(), **{k: v.numpy() for k, v in sd.items()}, "flat": flat.numpy()}
