"""The C-ABI library loads, exports every entry point include/moe_b200.h
declares, and rejects bad arguments before touching a GPU (CPU only)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from lightreason_b200 import build, native

HEADER = Path(__file__).resolve().parents[1] / "include" / "moe_b200.h"


def declared() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(moe_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def so():
    build.build()
    return native.lib()


def test_every_declared_symbol_is_exported(so):
    names = declared()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(so, n)]
    assert not missing, missing
    assert set(names) == set(native.EXPORTED), "native.py binds a different symbol set than the header declares"


def test_version_and_error_channel(so):
    assert so.moe_version() >= 100
    rc = so.moe_gather_rows(None, None, None, None, None, None, 1, 1, 1, 0, 1, 33, None)
    assert rc == native.MOE_EINVAL
    assert b"null table" in so.moe_last_error()
    with pytest.raises(ValueError):
        native.check(rc, "moe_gather_rows")


def test_argument_checks_precede_device_use(so):
    fake = ctypes.c_void_p(16)
    # threads not a multiple of 32
    assert so.moe_gather_rows(fake, fake, fake, fake, fake, fake, 1, 1, 1, 0, 1, 33, None) == native.MOE_EINVAL
    # unknown codec is rejected only after the checks that need no GPU; bad experts first
    assert so.moe_gather_rows(fake, fake, fake, fake, fake, fake, 0, 1, 1, 0, 1, 32, None) == native.MOE_EINVAL
    assert so.moe_permute(fake, 4, 8, 2048, fake, fake, fake, fake, fake, fake, None, None) == native.MOE_EINVAL
    assert so.moe_router_topk(fake, fake, None, None, 1, 3000, 256, 8, fake, fake, None, None, None,
                              None) == native.MOE_EINVAL
    assert so.moe_expert_rows(None, None, None, None, 129, None, 0, None) == native.MOE_EINVAL


def test_noalloc_argument_checks_precede_device_use(so):
    """The allocation-free expert rows refuse a table beyond their built-in
    128-pair array, and NULL token ids with more than one token, before any
    device call."""
    fake = ctypes.c_void_p(16)
    assert so.moe_expert_block_rows_noalloc(fake, fake, fake, fake, fake, 1, 129, None) == native.MOE_EINVAL
    assert b"built-in scratch" in so.moe_last_error()
    assert so.moe_expert_block_rows_noalloc(fake, fake, fake, None, fake, 2, 8, None) == native.MOE_EINVAL
    assert b"token_ids may be NULL only for one token" in so.moe_last_error()


def test_workspace_query_is_host_only(so):
    small = native.layer_workspace_bytes(1, 256, 8, 2048, 512)
    big = native.layer_workspace_bytes(4096, 256, 8, 2048, 512)
    assert 0 < small < big
    # y for T*K + T routes of 2048 BF16 dominates
    assert big >= (4096 * 9) * 2048 * 2


def test_layer_rejects_misaligned_rows_before_device_use(so):
    """Rows are read with 16-byte loads, TMA and bulk copies: a pointer off a
    16-byte boundary (say, a view that starts mid-row in a BF16 tensor) or an
    expert stride that is not a multiple of 8 elements is an argument error
    reported by the call, not a fault on the device."""
    good, bad = 1 << 20, (1 << 20) + 2
    ws = native.layer_workspace_bytes(1, 256, 8, 2048, 512)

    def call(x=good, out=good, **fields):
        w = native.LayerWeights(router=good, gate_up=good, down=good, experts=256, hidden=2048, inner=512,
                                top_k=8)
        for k, v in fields.items():
            setattr(w, k, v)
        return so.moe_layer_forward(ctypes.byref(w), ctypes.c_void_p(x), 1, ctypes.c_void_p(out), None,
                                    ctypes.c_void_p(good), ws, None)

    for kwargs in (dict(x=bad), dict(out=bad), dict(gate_up=bad), dict(down=bad), dict(router=bad),
                   dict(shared_gate=bad, shared_up=good, shared_down=good, shared_gate_w=good, shared_inner=512),
                   dict(gate_up_stride=2 * 512 * 2048 + 4)):
        assert call(**kwargs) == native.MOE_EINVAL, kwargs
        assert b"16-byte aligned" in so.moe_last_error(), kwargs


def test_empty_batch_is_a_no_op_before_device_use(so):
    """tokens == 0 is an empty batch, as the eager module takes it: the
    router, permute checks, layer, combine and shared-expert entry points
    return MOE_OK with NULL per-token arrays (an empty CUDA tensor's data
    pointer) and touch no device, while a bad shape in an empty batch is
    still an argument error."""
    good = ctypes.c_void_p(1 << 20)
    w = native.LayerWeights(router=1 << 20, gate_up=1 << 20, down=1 << 20, experts=256, hidden=2048, inner=512,
                            top_k=8)
    assert so.moe_layer_forward(ctypes.byref(w), None, 0, None, None, None, 0, None) == native.MOE_OK
    bad = native.LayerWeights(router=1 << 20, gate_up=1 << 20, down=1 << 20, experts=256, hidden=2048, inner=384,
                              top_k=8)
    assert so.moe_layer_forward(ctypes.byref(bad), None, 0, None, None, None, 0, None) == native.MOE_EINVAL
    assert so.moe_router_topk(None, good, None, None, 0, 2048, 256, 8, None, None, None, None, None,
                              None) == native.MOE_OK
    assert so.moe_router_topk(None, good, None, None, 0, 3000, 256, 8, None, None, None, None, None,
                              None) == native.MOE_EINVAL
    assert so.moe_router_select(None, None, 0, 256, 8, None, None, None, None) == native.MOE_OK
    assert so.moe_combine(None, None, None, None, None, 0, 8, 2048, None, None) == native.MOE_OK
    assert so.moe_combine(None, None, None, None, None, 0, 8, 2047, None, None) == native.MOE_EINVAL
    assert so.moe_shared_expert(None, good, good, good, None, 0, 2048, 512, None, None, None, 0,
                                None) == native.MOE_OK
