"""The update entry point that allocates nothing (memt_gdn2_update_noalloc).

Some callers cannot allocate device memory when they run the update: engines that size their
memory pool once at start-up, or FFI hosts without a caching allocator. This entry point takes
its scratch from a static 64 MiB device array instead of a caller workspace. These tests call
it through the C ABI and compare it with the allocating entry point (memt_gdn2_update, driven
by memt_b200.ops.gdn2_update with a torch-allocated workspace) on two calls in a row with
different inputs, so stale scratch from the first call cannot hide a fault in the second.
They must pass alone in a fresh process and after the rest of the suite.
"""

import ctypes

import numpy as np
import pytest
import torch

from memt_b200 import _lib, ops
from oracle import gdn2 as O

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-3  # the suite's bf16 tolerance (relative Frobenius)


def _inputs(seed, lengths, H, D, dev):
    gen = torch.Generator(device=dev).manual_seed(seed)
    L = sum(lengths)
    bf = torch.bfloat16

    def nrm(x):
        return (x / torch.sqrt((x ** 2).sum(-1, keepdim=True) + 1e-6)).to(bf)

    return dict(
        k=nrm(torch.randn(L, H, D, device=dev, generator=gen)),
        v=torch.randn(L, H, D, device=dev, generator=gen).to(bf),
        g=torch.nn.functional.logsigmoid(2.0 + 0.5 * torch.randn(L, H, D, device=dev, generator=gen)),
        beta=torch.sigmoid(torch.randn(L, H, device=dev, generator=gen)).to(bf),
        w=torch.sigmoid(torch.randn(L, H, D, device=dev, generator=gen)).to(bf),
        h0=0.02 * torch.randn(len(lengths), H, D, D, device=dev, generator=gen),
        cu=torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=dev),
    )


def _noalloc(x, lengths, H, D, out):
    args = _lib.UpdateArgs(
        num_samples=len(lengths), num_heads=H, key_dim=D, value_dim=D, total_tokens=sum(lengths),
        chunk_tokens=2048, dtype=_lib.MEMT_BF16, cu_seqlens=x["cu"].data_ptr(), k=x["k"].data_ptr(),
        v=x["v"].data_ptr(), g=x["g"].data_ptr(), g_layout=_lib.GATE_PER_CHANNEL, beta=x["beta"].data_ptr(),
        beta_layout=_lib.GATE_PER_HEAD, write=x["w"].data_ptr(), write_layout=_lib.GATE_PER_CHANNEL,
        initial_state=x["h0"].data_ptr(), final_state=out.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return _lib.load().memt_gdn2_update_noalloc(ctypes.byref(args), stream)


def test_noalloc_update_matches_allocating_entry(cuda):
    lengths, H, D = [300, 1, 129, 64], 4, 128
    for seed in (0, 1):  # two calls in a row
        x = _inputs(seed, lengths, H, D, cuda)
        ref = ops.gdn2_update(x["k"], x["v"], x["g"], x["h0"], x["cu"], num_samples=len(lengths),
                              total_tokens=sum(lengths), beta=x["beta"], write=x["w"])
        out = torch.full_like(x["h0"], float("nan"))
        _lib.check(_noalloc(x, lengths, H, D, out), "memt_gdn2_update_noalloc")
        torch.cuda.synchronize()
        err = O.rel_fro(out.cpu().numpy(), ref.cpu().numpy())
        assert err <= TOL_BF16, (seed, err)
        # the status word of the call, read from the static scratch by the library itself
        status = ctypes.c_int32(-1)
        _lib.check(_lib.load().memt_gdn2_noalloc_status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                                        ctypes.byref(status)), "memt_gdn2_noalloc_status")
        assert status.value == 0


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    lib = _lib.load()
    # 16 heads of 64k tokens need far more than the 64 MiB static scratch
    args = _lib.UpdateArgs(num_samples=1, num_heads=16, key_dim=128, value_dim=128, total_tokens=65536,
                           chunk_tokens=2048, dtype=_lib.MEMT_BF16, cu_seqlens=16, k=16, v=16, g=16,
                           g_layout=_lib.GATE_PER_HEAD, initial_state=16, final_state=16)
    need = lib.memt_gdn2_update_workspace_size(1, 65536, 16, 128, 128, 2048, _lib.MEMT_BF16)
    assert need > (64 << 20)
    assert lib.memt_gdn2_update_noalloc(ctypes.byref(args), None) == _lib.MEMT_ERR_WORKSPACE
