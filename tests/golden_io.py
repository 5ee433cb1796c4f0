"""Loads the golden fixtures written by tests/golden/make_golden.py."""
import json
from types import SimpleNamespace

import numpy as np

from conftest import GOLDEN

CASES = ["flex_5d_bf16_neox", "strict_5d_bf16_neox", "flex_5dpf_f16_gptj", "strict_4d_bf16_neox_partial"]
DT = {"bfloat16": "bf16", "float16": "f16", "float32": "f32"}


def load_case(name):
    meta = json.loads((GOLDEN / f"rerotate_{name}.json").read_text())
    arr = np.load(GOLDEN / f"rerotate_{name}.npz")
    return meta, {k: arr[k] for k in arr.files}


def contiguous_strides(shape):
    st, acc = [], 1
    for s in reversed(shape):
        st.append(acc)
        acc *= s
    return tuple(reversed(st))


def metas_of(meta):
    return [SimpleNamespace(ptr=p, saved_pos=s, block_ids=(b,))
            for p, s, b in zip(meta["ptr"], meta["saved_pos"], meta["block_ids"])]


def policy_cases():
    return json.loads((GOLDEN / "policy_cases.json").read_text())
