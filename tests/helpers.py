"""Shared checks for the parity tests: the tolerances of the north-star
contract (max-abs 2e-2 and rel-L2 1e-2 on BF16 outputs with FP32 accumulation)
and the two-tier rule for expert ids."""

from __future__ import annotations

from pathlib import Path

import numpy as np

from lightreason_b200 import synthetic as S

GOLDEN = Path(__file__).resolve().parent / "golden"
MAX_ABS = 2e-2
REL_L2 = 1e-2
# tier-2 near-tie tokens per case, printed in the pytest terminal summary so a
# change in the router's summation order shows as a change in these counts
EXCUSED: dict[str, tuple[int, int]] = {}


def f32(bits) -> np.ndarray:
    return S.bf16_bits_to_f32(np.asarray(bits))


def assert_close(got_bits, want_bits, *, max_abs=MAX_ABS, rel_l2=REL_L2, what="output"):
    got, want = f32(got_bits).astype(np.float64), f32(want_bits).astype(np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite values"
    err = np.abs(got - want).max() if got.size else 0.0
    rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    assert err <= max_abs, f"{what}: max-abs {err:.3e} > {max_abs}"
    assert rel <= rel_l2, f"{what}: rel-L2 {rel:.3e} > {rel_l2}"
    return err, rel


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    """One BF16 ulp at |x| (FP32 result)."""
    x = np.abs(np.asarray(x, dtype=np.float32))
    exp = np.floor(np.log2(np.maximum(x, np.float32(2.0 ** -126))))
    return (2.0 ** (exp - 7)).astype(np.float32)


def compare_ids(got: np.ndarray, want: np.ndarray, z_ref: np.ndarray, *, slack_ulps: float = 0.0,
                case: str | None = None):
    """Tier-2 id parity.  Rows must match exactly, except where the reference's
    own z (= logits + bias) has a near tie at the boundary that moved: the
    selections may then differ only among experts whose z lies within
    `slack_ulps` BF16 ulps of the k-th largest.  Returns the number of tokens
    that needed the slack (recorded under `case` for the session summary).
    With slack 0 an exact tie is compared as a set."""
    got, want = np.asarray(got), np.asarray(want)
    assert got.shape == want.shape
    k = got.shape[1]
    excused = 0
    for t in range(got.shape[0]):
        if np.array_equal(got[t], want[t]):
            continue
        z = z_ref[t]
        kth = np.sort(z)[::-1][k - 1]
        tol = slack_ulps * bf16_ulp(kth) if slack_ulps else 0.0
        sg, sw = set(got[t].tolist()), set(want[t].tolist())
        diff = sg ^ sw
        assert all(abs(z[e] - kth) <= tol for e in diff), (
            f"token {t}: ids {got[t]} vs {want[t]} differ beyond a near tie")
        # the common ids must keep the reference's order up to ties
        common = [e for e in want[t] if e in sg]
        zc = z[common]
        assert np.all(np.diff(zc) <= tol), f"token {t}: order differs beyond ties"
        excused += 1
    if case is not None:
        EXCUSED[case] = (excused, int(got.shape[0]))
    return excused


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / name, allow_pickle=False) as f:
        return {k: f[k] for k in f.files}


def golden_layers():
    return sorted(p.name for p in GOLDEN.glob("layer_T*_s*.npz"))
