"""GPU parity of the DeepSeek (Flash) memory block's projections around the GDN-2 path:
the grouped latent RMS norm kernel, the grouped low-rank q/k/v expansion, the gate and q/k
preparation in the prologue kernel (rsqrt l2norm) and the wo_a memory injection. Compared with
the reference's own eager outputs (tests/golden/flash_projections.npz) and with the oracle.
bf16 results: relative Frobenius <= 4e-3 (bf16 rounding of sums taken in another order, as for
the reference's own bf16 readout pipeline); fp32 log-decay <= 1e-6.
"""

import numpy as np
import pytest
import torch

from memt_b200 import flash
from oracle import gdn2 as O

pytestmark = pytest.mark.gpu

TOL_BF16_OUT = 4e-3


def _t(x, dev, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(np.asarray(x, np.float32))).to(dev).to(dtype)


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("T,G,R", [(1, 1, 8), (37, 2, 64), (300, 4, 512), (129, 1, 1536)])
def test_latent_rms_norm_matches_oracle(cuda, T, G, R):
    rng = np.random.default_rng(T + G + R)
    x = O.bf16(rng.standard_normal((T, G * R)) * 3.0)
    w = O.bf16(1.0 + 0.1 * rng.standard_normal((G, R)))
    eps = [1e-6 * (g + 1) for g in range(G)]
    # a strided view: the latent as columns of a wider projection output
    wide = torch.zeros(T, G * R + 24, device=cuda, dtype=torch.bfloat16)
    wide[:, 8:8 + G * R] = _t(x, cuda)
    got = flash.latent_rms_norm(wide[:, 8:8 + G * R], _t(w, cuda), eps)
    torch.cuda.synchronize()
    ref = O.latent_rms_norm(x.reshape(T, G, R), w, eps)
    assert got.shape == (T, G, R)
    assert O.rel_fro(_np(got), ref) <= 2e-3


def test_flash_projections_match_reference(golden, cuda):
    z = golden("flash_projections")
    G, H, D = int(z["groups"]), int(z["heads"]), int(z["head_dim"])
    eps = float(z["eps"])
    q, k, v = flash.expand_grouped_qkv(_t(z["q_lat"], cuda), _t(z["k_lat"], cuda), _t(z["v_lat"], cuda),
                                       _t(z["q_norm"], cuda), _t(z["q_up"], cuda), eps, _t(z["k_up"], cuda),
                                       _t(z["v_up"], cuda), _t(z["k_norm"], cuda), _t(z["v_norm"], cuda),
                                       (eps,) * G, (eps,) * G)
    T = z["q"].shape[0]
    query, key, write, log_decay = flash.head_inputs(
        _t(z["q"], cuda).view(T, H, D), _t(z["k"], cuda).view(T, H, D), _t(z["erase_gate"], cuda),
        _t(z["write_gate"], cuda), _t(z["decay_latent"], cuda), _t(z["decay_bias"], cuda),
        _t(z["decay_scale_log"], cuda))
    torch.cuda.synchronize()
    for got, ref in ((q, z["q"]), (k, z["k"]), (v, z["v"])):
        assert O.rel_fro(_np(got), ref) <= TOL_BF16_OUT
    for got, ref in ((query, z["query"]), (key, z["key"]), (write, z["write"])):
        assert O.rel_fro(_np(got[0]), ref) <= TOL_BF16_OUT
    assert O.rel_fro(_np(log_decay[0]), z["log_decay"]) <= 1e-6


@pytest.mark.parametrize("T,G,d,r", [(1, 1, 64, 32), (300, 4, 512, 128), (65, 8, 2048, 1024)])
def test_memory_inject_matches_oracle(cuda, T, G, d, r):
    rng = np.random.default_rng(T + G)
    mem = O.bf16(rng.standard_normal((T, G * d)))
    wo_a = O.bf16(rng.standard_normal((G * r, d)) * d ** -0.5)
    res = O.bf16(rng.standard_normal((T, G * r)))
    out = _t(res, cuda)
    ptr = out.data_ptr()
    got = flash.memory_inject(_t(mem, cuda), _t(wo_a, cuda), G, out)
    torch.cuda.synchronize()
    assert got.data_ptr() == ptr  # in place
    ref = O.memory_inject(mem, wo_a, G, res)
    assert O.rel_fro(_np(got), ref) <= TOL_BF16_OUT
