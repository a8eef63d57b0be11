"""The allocation-free expert-rows entry point (GPU only).

moe_expert_block_rows_noalloc serves callers that hold only device pointers
and may not allocate device memory themselves (a native worker standing in for
the reference's cpu_experts.c call, or a server that forbids allocation while
it runs): its intermediate activations live in a fixed array inside the
library.  This file checks it, through the C ABI, against the workspace entry
point moe_expert_block_rows on consecutive calls -- each later call finds the
earlier call's leftovers in the shared array -- including a table of exactly
128 pairs, which fills the array to its last byte.  Both entry points run the
same kernels in the same order, so the outputs must be bit-identical.  Tables
larger than the built-in array are refused.  It is collected last and sets
itself up, so it passes alone in a fresh process as well as after the other
tests.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from lightreason_b200 import build, native
from lightreason_b200 import synthetic as S

pytestmark = pytest.mark.gpu


def _dev(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(dev).view(torch.bfloat16)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _noalloc(lib, gate_up, down, hidden, token_ids, out):
    pairs = len(gate_up)
    gp = (ctypes.c_void_p * pairs)(*[t.data_ptr() for t in gate_up])
    dp = (ctypes.c_void_p * pairs)(*[t.data_ptr() for t in down])
    tid = None if token_ids is None else ctypes.cast((ctypes.c_int32 * pairs)(*token_ids), ctypes.c_void_p)
    rc = lib.moe_expert_block_rows_noalloc(ctypes.cast(gp, ctypes.c_void_p), ctypes.cast(dp, ctypes.c_void_p),
                                           hidden.data_ptr(), tid, out.data_ptr(), hidden.shape[0], pairs,
                                           torch.cuda.current_stream().cuda_stream)
    native.check(rc, "moe_expert_block_rows_noalloc")


def test_noalloc_rows_match_workspace_entry_point_on_consecutive_calls():
    build.build()
    lib = native.lib()
    native.device_check(0)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(2024)
    w = S.layer_weights(21)
    experts = rng.choice(S.EXPERTS, size=6, replace=False)
    w.ensure(experts)
    gu_dev = {e: _dev(w.gate_up[e], dev) for e in experts}
    dn_dev = {e: _dev(w.down[e], dev) for e in experts}
    # calls in a row with different tables: 24 pairs over 5 tokens, 9 pairs
    # over 3, then the largest table (128 pairs over 16 tokens, the whole array)
    for call, (pairs, tokens) in enumerate(((24, 5), (9, 3), (128, 16))):
        pair_experts = rng.choice(experts, size=pairs)
        token_ids = rng.integers(0, tokens, size=pairs).tolist()
        gu = [gu_dev[e] for e in pair_experts]
        dn = [dn_dev[e] for e in pair_experts]
        x = _dev(S.hidden_states(30 + call, tokens), dev)
        want = native.expert_block_rows(gu, dn, x, token_ids)
        got = torch.full_like(want, 7.0)
        _noalloc(lib, gu, dn, x, token_ids, got)
        torch.cuda.synchronize()
        assert np.array_equal(_bits(got), _bits(want)), f"noalloc call {call}: output differs from the workspace path"
    # one token, no token ids: the expert_rows form
    gu = [gu_dev[e] for e in experts]
    dn = [dn_dev[e] for e in experts]
    x1 = _dev(S.hidden_states(40, 1), dev)
    want = native.expert_block_rows(gu, dn, x1)
    got = torch.empty_like(want)
    _noalloc(lib, gu, dn, x1, None, got)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(got), _bits(want)), "noalloc expert_rows form differs from the workspace path"


def test_noalloc_rejects_tables_beyond_its_scratch():
    build.build()
    lib = native.lib()
    null = ctypes.c_void_p(0)
    rc = lib.moe_expert_block_rows_noalloc(null, null, null, null, null, 1, 129, None)
    assert rc == native.MOE_EINVAL
    assert b"built-in scratch" in lib.moe_last_error()
