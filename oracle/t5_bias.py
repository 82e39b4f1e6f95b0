"""CPU restatement of the T5 relative-position bias that feeds the T5 attention call site.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): never imported by the product.

relative_bucket follows app/models/t5.js:14-23, which restates Hugging Face transformers'
T5Attention._relative_position_bucket (bidirectional) in float32 with Math.fround at every
step; here numpy float32 scalars give the same rounding. position_bias follows
app/models/t5.js:55-65: out[(h*L + i)*L + j] = table[bucket(j - i)*H + h].
"""

from __future__ import annotations

import math

import numpy as np


def relative_bucket(rel: int, buckets: int = 32, max_distance: int = 128) -> int:
    """app/models/t5.js:14-23 (bidirectional bucket of rel = key - query)."""
    nb = buckets // 2
    bucket = nb if rel > 0 else 0
    n = abs(int(rel))
    max_exact = nb // 2
    if n < max_exact:
        return bucket + n
    f = np.float32
    a = f(n / max_exact)                      # Math.fround(n / maxExact)
    b = f(math.log(float(a)))                 # Math.fround(Math.log(...)) (double log)
    c = f(math.log(max_distance / max_exact))  # Math.fround(Math.log(maxDistance / maxExact))
    d = f(float(b) / float(c))                # fround of the division
    e = f(float(d) * (nb - max_exact))        # fround of the product
    large = max_exact + math.trunc(float(e))
    return bucket + min(large, nb - 1)


def relative_bucket_table(L: int, buckets: int = 32, max_distance: int = 128) -> np.ndarray:
    """Buckets for rel = -(L-1) .. L-1 (index rel + L - 1), int32."""
    return np.array([relative_bucket(r, buckets, max_distance) for r in range(-(L - 1), L)], dtype=np.int32)


def position_bias(table, L: int, H: int, buckets: int = 32, max_distance: int = 128) -> np.ndarray:
    """T5Encoder.positionBias(L) (app/models/t5.js:55-65): flat float32 [H, L, L].

    table is [buckets, H] (encoder.block.0...relative_attention_bias.weight, app/models/t5.js:44).
    """
    t = np.asarray(table, dtype=np.float32).reshape(buckets, H)
    lut = relative_bucket_table(L, buckets, max_distance)
    i = np.arange(L)[:, None]
    j = np.arange(L)[None, :]
    bk = lut[(j - i) + L - 1]                # [L, L] bucket of (j - i)
    return np.ascontiguousarray(t[bk].transpose(2, 0, 1)).reshape(-1)  # [H, L, L]
