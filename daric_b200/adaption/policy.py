"""DARIC recompute-budget policy (host side).

Restates ``DARICPolicy`` / ``cluster_groups`` of the reference
(daric/adaption/policy.py:5-103) so that the recompute ranges are identical:
the budget ``avg_num * num_groups`` is spread over the heads of the reused
groups as ``round(a * f(i) + b)`` tokens (Python round, half to even), with
a, b and the tail length solved from a 3x3 fp32 system by
``torch.linalg.solve`` (policy.py:61-72), a tail run before the last token,
and two rebalancing passes (policy.py:92-103). Its ranges are expanded into
positions and slots on the GPU by ``daric_b200.select.ptrs_to_slots``.
"""
from __future__ import annotations

import math

import torch

__all__ = ["DARICPolicy", "cluster_groups"]


def cluster_groups(ranges):
    """Merges consecutive [start, end) ranges whose start is not past the
    current end (policy.py:5-14)."""
    merged = []
    cur = list(ranges[0])
    for start, end in ranges[1:]:
        if start > cur[1]:
            merged.append(cur)
            cur = [start, end]
        else:
            cur = [min(start, cur[0]), max(cur[1], end)]
    merged.append(cur)
    return merged


def _linear(x, r=1):
    return r * x


def _exp(x, r=0.2):
    return math.exp(r * x)


def _log(x, r=0.2):
    return math.log(r * x)


_FUNCTIONS = {"linear": _linear, "exp": _exp, "log": _log}


class DARICPolicy:
    def __init__(self, avg_num: int = 32, r: float = 0.1, function: str = "linear"):
        if function not in _FUNCTIONS:
            raise ValueError(f"Unknown function: {function}")
        self.alpha = 1  # the weight function is evaluated as f(i, alpha)
        self.r = r
        self.avg_num = avg_num
        self.function = _FUNCTIONS[function]

    def get_recompute_ptrs(self, group_ptr: list[int]) -> list[list[int]]:
        n_groups = len(group_ptr) - 1
        budget = self.avg_num * n_groups
        if n_groups == 1:
            return []
        if n_groups == 2:
            half = int(budget / 2)
            return cluster_groups([
                [group_ptr[1], min(group_ptr[1] + half, group_ptr[2])],
                [max(0, group_ptr[2] - half), group_ptr[2] - 1],
            ])
        f = self.function
        f_first = f(1, self.alpha)
        f_last = f(n_groups - 1, self.alpha)
        f_total = sum(f(i, self.alpha) for i in range(1, n_groups))
        system = torch.tensor([[f_last, 1, -1], [f_first, 1, 0], [f_total, n_groups - 1, 1]]).float()
        rhs = torch.tensor([0, self.r * self.avg_num, budget], dtype=torch.float32)
        a, b, tail = torch.linalg.solve(system, rhs).tolist()

        ranges = []
        for i in range(1, n_groups):
            count = max(1, round(a * f(i, self.alpha) + b))
            ranges.append([group_ptr[i], min(group_ptr[i] + count, group_ptr[i + 1])])
        if ranges[-1][1] == group_ptr[-1]:
            ranges[-1][1] -= 1
        else:
            tail_count = round(tail)
            if tail_count > 1:
                ranges.append([max(0, group_ptr[-1] - 1 - tail_count), group_ptr[-1] - 1])
        ranges = cluster_groups(ranges)
        left = budget - sum(e - s for s, e in ranges)
        for _ in range(2):
            ranges[-1][0] = max(0, ranges[-1][0] - left)
            ranges = cluster_groups(ranges)
            left = budget - sum(e - s for s, e in ranges)
            if left == 0:
                break
        return ranges
