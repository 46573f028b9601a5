"""C ABI checks that need no GPU: the library loads, exports every declared symbol, and
rejects bad arguments on the host before touching CUDA."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from memt_b200 import _lib
from memt_b200.layout import build_chunk_plan, packed_plan
from oracle import gdn2 as O

HEADER = Path(__file__).resolve().parents[1] / "include" / "memt_gdn2.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(memt_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 9
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures must cover the header"


def test_version_and_status_strings():
    lib = _lib.load()
    assert lib.memt_version() >= 100
    assert lib.memt_status_string(0) == b"ok"
    assert b"workspace" in lib.memt_status_string(-4)


def _cu(lengths):
    return (ctypes.c_int32 * (len(lengths) + 1))(*np.concatenate([[0], np.cumsum(lengths)]).astype(int))


@pytest.mark.parametrize("lengths,ct", [([512], 2048), ([100, 37, 64, 1, 65, 130], 128), ([8192] * 8, 2048),
                                        ([300, 5], 100), ([1, 2, 3], 1)])
def test_count_chunks_matches_oracle_plan(lengths, ct):
    lib = _lib.load()
    cu = np.concatenate([[0], np.cumsum(lengths)])
    assert lib.memt_gdn2_count_chunks(_cu(lengths), len(lengths), ct) == len(O.plan_chunks(cu, ct))


def test_count_chunks_rejects_bad_offsets():
    lib = _lib.load()
    bad = (ctypes.c_int32 * 3)(0, 10, 5)
    assert lib.memt_gdn2_count_chunks(bad, 2, 64) == -1
    assert lib.memt_gdn2_count_chunks(_cu([4]), 1, 0) == -1


def test_workspace_size():
    lib = _lib.load()
    f = lib.memt_gdn2_update_workspace_size
    assert f(8, 65536, 16, 128, 128, 2048, _lib.MEMT_BF16) > 3 * 65536 * 16 * 128 * 2
    assert f(1, 512, 4, 64, 64, 2048, _lib.MEMT_F32) == 256
    assert f(1, 512, 4, 96, 96, 2048, _lib.MEMT_BF16) == 0   # unsupported head dim
    assert f(1, 512, 4, 64, 128, 2048, _lib.MEMT_BF16) == 0  # K != V
    assert f(0, 512, 4, 64, 64, 2048, _lib.MEMT_BF16) == 0


def test_update_rejects_bad_arguments_before_launch():
    lib = _lib.load()
    assert lib.memt_gdn2_update(None, None, 0, None) == _lib.MEMT_ERR_INVALID_ARGUMENT
    a = _lib.UpdateArgs(num_samples=1, num_heads=1, key_dim=64, value_dim=64, total_tokens=4, chunk_tokens=64,
                        dtype=_lib.MEMT_BF16, cu_seqlens=16, k=16, v=16, g=16, g_layout=_lib.GATE_PER_HEAD,
                        initial_state=16, final_state=16)
    # missing workspace
    assert lib.memt_gdn2_update(ctypes.byref(a), None, 0, None) == _lib.MEMT_ERR_WORKSPACE
    a.key_dim = a.value_dim = 96
    assert lib.memt_gdn2_update(ctypes.byref(a), None, 0, None) == _lib.MEMT_ERR_UNSUPPORTED
    a.key_dim = a.value_dim = 64
    a.k = 18  # misaligned
    assert lib.memt_gdn2_update(ctypes.byref(a), None, 0, None) == _lib.MEMT_ERR_MISALIGNED
    a.k = 16
    a.beta_layout = _lib.GATE_PER_HEAD  # layout without a pointer
    assert lib.memt_gdn2_update(ctypes.byref(a), None, 0, None) == _lib.MEMT_ERR_INVALID_ARGUMENT
    a.beta_layout = 0
    a.g_layout = 7
    assert lib.memt_gdn2_update(ctypes.byref(a), None, 0, None) == _lib.MEMT_ERR_INVALID_ARGUMENT


def test_read_and_readout_reject_bad_arguments():
    lib = _lib.load()
    assert lib.memt_gdn2_read(None, None) == _lib.MEMT_ERR_INVALID_ARGUMENT
    r = _lib.ReadArgs(num_blocks=1, num_heads=1, key_dim=128, value_dim=128, total_tokens=1, cu_seqlens=16, q=16,
                      q_dtype=_lib.MEMT_BF16, states=16, scale=0.1, out=16, out_dtype=9)
    assert lib.memt_gdn2_read(ctypes.byref(r), None) == _lib.MEMT_ERR_INVALID_ARGUMENT
    assert lib.memt_memory_readout(None, None) == _lib.MEMT_ERR_INVALID_ARGUMENT
    ro = _lib.ReadoutArgs(num_blocks=1, num_heads=2, head_dim=128, total_tokens=1, cu_seqlens=16, q=16,
                          states=16, gate=16, norm_weight=16, out=16, row_stride=128)
    assert lib.memt_memory_readout(ctypes.byref(ro), None) == _lib.MEMT_ERR_INVALID_ARGUMENT  # row too short


@pytest.mark.parametrize("lengths,ct", [([100, 37, 64, 1, 65, 130], 128), ([512], 2048), ([200, 3], 64)])
def test_host_plan_matches_oracle(lengths, ct):
    plan = packed_plan(lengths, "cpu", chunk_tokens=ct)
    cu = np.concatenate([[0], np.cumsum(lengths)])
    chunks = O.plan_chunks(cu, ct)
    assert plan.num_chunk == len(chunks)
    assert plan.chunk_tok0.tolist() == [t0 for _, t0, _ in chunks]
    assert plan.chunk_len.tolist() == [ln for _, _, ln in chunks]
    assert plan.chunk_block_ids.tolist() == [n for n, _, _ in chunks]
    assert plan.read_slice.tolist() == cu.tolist()
    assert plan.max_block_tokens == max(lengths)


def test_query_plan_has_one_block_per_sample():
    samples = torch.tensor([0, 1, 2, 7], dtype=torch.int32)
    plan = build_chunk_plan(samples, samples, event_slice=samples, commit_mask=torch.zeros(3, dtype=torch.bool))
    assert plan.num_block == 3 and plan.num_chunk == 3
    assert not plan.chunk_commits.any()
    assert plan.max_block_tokens == 5


def test_argument_structs_carry_their_size():
    """Every argument struct starts with struct_size; a struct of another size (for example a
    binding written against the 0.2 layout, whose first field is num_samples) is rejected
    before anything is read or launched."""
    lib = _lib.load()
    assert lib.memt_version() == 300
    a = _lib.UpdateArgs(num_samples=1, num_heads=1, key_dim=64, value_dim=64, total_tokens=4, chunk_tokens=64,
                        dtype=_lib.MEMT_BF16, cu_seqlens=16, k=16, v=16, g=16, g_layout=_lib.GATE_PER_HEAD,
                        initial_state=16, final_state=16)
    assert a.struct_size == ctypes.sizeof(_lib.UpdateArgs)
    # the right size gets past the struct check (the missing workspace is the next error)
    assert lib.memt_gdn2_update(ctypes.byref(a), None, 0, None) == _lib.MEMT_ERR_WORKSPACE
    for size in (0, ctypes.sizeof(_lib.UpdateArgs) - 24, ctypes.sizeof(_lib.UpdateArgs) + 8):
        a.struct_size = size
        assert lib.memt_gdn2_update(ctypes.byref(a), None, 0, None) == _lib.MEMT_ERR_INVALID_ARGUMENT
        assert lib.memt_gdn2_update_noalloc(ctypes.byref(a), None) == _lib.MEMT_ERR_INVALID_ARGUMENT

    class UpdateArgsV02(ctypes.Structure):  # the 0.2.0 layout: no struct_size
        _fields_ = [(name, typ) for name, typ in _lib.UpdateArgs._fields_ if name != "struct_size"]

    old = UpdateArgsV02(num_samples=8, num_heads=16, key_dim=128, value_dim=128, total_tokens=65536,
                        chunk_tokens=2048, dtype=_lib.MEMT_BF16)
    assert lib.memt_gdn2_update(ctypes.cast(ctypes.byref(old), ctypes.POINTER(_lib.UpdateArgs)), None, 0,
                                None) == _lib.MEMT_ERR_INVALID_ARGUMENT
    r = _lib.ReadArgs(num_blocks=1, num_heads=1, key_dim=128, value_dim=128, total_tokens=0, cu_seqlens=16, q=16,
                      q_dtype=_lib.MEMT_BF16, states=16, scale=0.1, out=16, out_dtype=_lib.MEMT_BF16)
    assert lib.memt_gdn2_read(ctypes.byref(r), None) == _lib.MEMT_OK  # no tokens: nothing to launch
    r.struct_size -= 8
    assert lib.memt_gdn2_read(ctypes.byref(r), None) == _lib.MEMT_ERR_INVALID_ARGUMENT
    ro = _lib.ReadoutArgs(num_blocks=1, num_heads=1, head_dim=128, total_tokens=0, cu_seqlens=16, q=16,
                          states=16, gate=16, norm_weight=16, out=16, row_stride=128)
    assert lib.memt_memory_readout(ctypes.byref(ro), None) == _lib.MEMT_OK
    ro.struct_size = 4
    assert lib.memt_memory_readout(ctypes.byref(ro), None) == _lib.MEMT_ERR_INVALID_ARGUMENT
    p = _lib.PrologueArgs(num_heads=1, head_dim=64, total_tokens=0, q=16, q_stride=64, k=16, k_stride=64,
                          erase_latent=16, erase_stride=64, write_latent=16, write_stride=64, decay_latent=16,
                          decay_stride=64, decay_bias=16, decay_scale_log=16, q_out=16, k_out=16, write_out=16,
                          log_decay_out=16)
    assert lib.memt_qwen_prologue(ctypes.byref(p), None) == _lib.MEMT_OK
    p.q_stride = 60  # shorter than a token row
    assert lib.memt_qwen_prologue(ctypes.byref(p), None) == _lib.MEMT_ERR_INVALID_ARGUMENT
    p.q_stride = 68  # not a 16-byte multiple
    assert lib.memt_qwen_prologue(ctypes.byref(p), None) == _lib.MEMT_ERR_MISALIGNED
    p.q_stride = 64
    p.struct_size += 8
    assert lib.memt_qwen_prologue(ctypes.byref(p), None) == _lib.MEMT_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("lengths,ct", [([100, 37, 64, 1, 65, 130], 128), ([300, 5], 100), ([1], 1)])
def test_read_segments_of_a_plan(lengths, ct):
    """The read blocks memt_gdn2_read_fwd derives from a plan without read_slice (the
    reference's own ChunkPlan) are the samples, in order."""
    plan = packed_plan(lengths, "cpu", chunk_tokens=ct)
    from memt_b200.layout import read_segments
    cu, ids, longest = read_segments(plan)
    assert cu == np.concatenate([[0], np.cumsum(lengths)]).tolist()
    assert ids == list(range(len(lengths))) and longest == max(lengths)
