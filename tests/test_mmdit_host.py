"""Host-side pieces of the synthetic MMDiT (tfimage.mmdit) on the CPU: RoPE ids and tables against the oracle's
restatement (itself pinned to the reference), the sampler's sigmas, and the block oracle's attention."""

import math

import numpy as np
import torch

from oracle import dit as odit
from oracle import fusions
from tfimage import mmdit


def test_rope_tables_match_oracle_at_configs2_grid():
    cfg = mmdit.DitConfig()
    ids_t = mmdit.text_ids(256, "cpu")
    ids_i = mmdit.image_ids(64, 64, 256, "cpu")
    assert np.array_equal(ids_t.numpy(), fusions.text_ids(256))
    assert np.array_equal(ids_i.numpy(), fusions.image_ids(64, 64, 256, (64, 64)))
    for ids in (ids_t, ids_i):
        c, s = mmdit.rope_table(ids, cfg)
        rc, rs = fusions.rope_table(ids.numpy())
        assert np.array_equal(c.numpy(), rc) and np.array_equal(s.numpy(), rs)


def test_sigmas_shifted_simple_schedule():
    sig = mmdit.sigmas(25)
    assert len(sig) == 26 and sig[0] == 1.0 and sig[-1] == 0.0
    assert all(a > b for a, b in zip(sig, sig[1:]))
    t = 1 - 24 * 400 / 10000                                 # step 24 of 25 on the 10000-entry table
    expect = math.exp(mmdit.SHIFT) / (math.exp(mmdit.SHIFT) + (1 / np.float32(t) - 1))
    assert abs(sig[24] - expect) < 1e-6


def test_oracle_attention_causal_and_prefix():
    g = torch.Generator().manual_seed(3)
    q = torch.randn((1, 5, 2, 8), generator=g).numpy()
    k = torch.randn((1, 7, 2, 8), generator=g).numpy()
    v = torch.randn((1, 7, 2, 8), generator=g).numpy()
    full = odit.attention(q, k, v)
    ref = torch.nn.functional.scaled_dot_product_attention(
        *(torch.from_numpy(t).double().transpose(1, 2) for t in (q, k, v))).transpose(1, 2).float().numpy()
    assert np.abs(full - ref).max() <= 2 ** -7 * np.abs(ref).max()
    causal = odit.attention(q, k, v, causal=True)            # 2 prefix keys, then query i sees keys 0..2+i
    last = odit.attention(q[:, 4:], k, v)                    # the last query sees every key
    assert np.array_equal(causal[:, 4:], last)
    first = odit.attention(q[:, :1], k[:, :3], v[:, :3])
    assert np.array_equal(causal[:, :1], first)
