"""Pins the oracle and the host policy to golden vectors produced by the
reference itself (tests/golden/make_golden.py)."""
import numpy as np
import pytest

from golden_io import CASES, DT, contiguous_strides, load_case, metas_of, policy_cases
from oracle import rerotate as R


def test_policy_matches_reference_golden():
    from daric_b200.adaption.policy import DARICPolicy
    cases = policy_cases()
    assert len(cases) > 300
    for c in cases:
        pol = DARICPolicy(c["avg_num"], r=c["r"], function=c["function"])
        if "error" in c:
            with pytest.raises(Exception):
                pol.get_recompute_ptrs(c["group_ptr"])
            continue
        assert pol.get_recompute_ptrs(c["group_ptr"]) == c["ptrs"], c


def _run_oracle(meta, arr, rounding):
    dt = DT[meta["dtype"]]
    layer = R.KLayer(arr["kv_in"].reshape(-1).copy(), tuple(meta["shape"]), contiguous_strides(meta["shape"]),
                     meta["page_first"], dt)
    rot = R.Rotary(arr["table"].reshape(meta["max_pos"], meta["rotary_dim"]), dt, meta["rotary_dim"],
                   meta["is_neox"])
    name = meta["layer"]
    if meta["mode"] == "flexible":
        R.apply_rerotate_load({name: layer}, {name: rot}, {name: 0}, metas_of(meta), rounding=rounding)
    else:
        R.apply_rerotate_multi({name: layer}, {name: rot}, {name: 0}, meta["group_ptrs"],
                               [(b,) for b in meta["block_ids"]], rounding=rounding)
    return layer.raw


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_kernel(case):
    """The Triton interpreter truncates fp32->bf16; with the same cast the
    oracle reproduces the reference kernel bit for bit, and with RTNE (the
    GPU cast) it stays within 1 ulp of it."""
    meta, arr = load_case(case)
    dt = DT[meta["dtype"]]
    gold = arr["kv_out"].reshape(-1)
    assert not np.array_equal(gold, arr["kv_in"].reshape(-1)), "fixture rotated nothing"
    exact = _run_oracle(meta, arr, "trunc")
    np.testing.assert_array_equal(exact, gold)
    rtne = _run_oracle(meta, arr, "rtne")
    assert R.ulp_diff(rtne, gold, dt).max() <= 1
