"""Small shared helpers: timing decorators, project dir, best-fit segment tree.

Parity: reference ``pluggy/utils.py:11-80`` (``record_time``, ``debug_time``,
``get_project_dir``, ``Node``).

``record_time`` keeps the reference's host-clock contract (synchronize on both
sides, return ``(result, seconds)``) because the trainer's step line is built on
it. Benchmarks use :func:`pluggy_b200.utils.timing.device_time` instead: CUDA
events on the launching stream, max over ranks.
"""

from __future__ import annotations

import os
import time

import torch


def record_time(func):
    def wrapper(*args, **kwargs):
        cuda = torch.cuda.is_available()
        if cuda:
            torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = func(*args, **kwargs)
        if cuda:
            torch.cuda.synchronize()
        return out, time.perf_counter() - t0
    wrapper.__name__ = func.__name__
    wrapper.__doc__ = func.__doc__
    return wrapper


def debug_time(func):
    def wrapper(*args, **kwargs):
        t0 = time.perf_counter()
        out = func(*args, **kwargs)
        if os.environ.get("RANK", "0") == "0":
            print(f"{func.__name__} took {time.perf_counter() - t0} seconds to run")
        return out
    wrapper.__name__ = func.__name__
    return wrapper


def get_project_dir() -> str:
    return os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


class Node:
    """Max segment tree over free-space buckets ``[low, high]``.

    Leaf ``s`` holds ``s`` while some open bin has exactly ``s`` slots free, else
    0; ``search(c)`` returns the smallest bucket ``>= c`` that is available
    (best fit) in O(log n).
    """

    __slots__ = ("low", "high", "value", "left", "right")

    def __init__(self, low: int, high: int, value: int = 0):
        self.low, self.high, self.value = low, high, value
        self.left = self.right = None

    @classmethod
    def build(cls, low: int, high: int) -> "Node":
        node = cls(low, high)
        if low < high:
            mid = (low + high) // 2
            node.left = cls.build(low, mid)
            node.right = cls.build(mid + 1, high)
        return node

    def search(self, size: int):
        if self.value < size:
            return None
        node = self
        while node.low != node.high:
            node = node.left if node.left.value >= size else node.right
        return node.low

    def update(self, capacity: int, available: bool) -> None:
        if self.low == self.high:
            self.value = capacity if available else 0
            return
        (self.left if capacity <= self.left.high else self.right).update(capacity, available)
        self.value = max(self.left.value, self.right.value)
