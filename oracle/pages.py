"""TEST INFRASTRUCTURE ONLY — byte-exact restatement of the reference's page
gather/scatter (csrc/cache_ops/kernels.cu:7-45, 86-123) and of the shape
derivation and checks that precede it (helpers.cu:22-174, copier.cpp:32-39,
kernels.cu:151-161). Layers are numpy byte buffers with element sizes and
strides, so any tensor layout the reference accepts can be replayed.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


class OracleError(RuntimeError):
    pass


def _check(cond, msg):
    if not cond:
        raise OracleError(msg)


@dataclass
class LayerMem:
    """A KV layer: raw bytes (1-D uint8), sizes/strides in elements, element size."""
    mem: np.ndarray
    sizes: tuple
    strides: tuple
    es: int
    page_first: bool


def dense_span(sizes, strides, first) -> int:
    """helpers.cu:22-64: non-singleton dims from `first`, sorted by stride,
    must be densely packed; returns the element span."""
    dims = []
    for d in range(first, len(sizes)):
        _check(sizes[d] > 0, "KV cache copy dimensions must be non-empty")
        if sizes[d] == 1:
            continue
        _check(strides[d] > 0, "KV cache non-singleton dimensions must have positive strides")
        dims.append((strides[d], sizes[d], d))
    dims.sort(key=lambda t: t[0])
    expect = 1
    for stride, size, _ in dims:
        _check(stride == expect, "KV cache copy dimensions must form a dense physical span")
        expect *= size
    return expect


def page_copy_shape(sizes, strides, es, page_first):
    """helpers.cu:94-148 -> (num_pages, prefix_size, page_stride, suffix, prefix_stride), bytes."""
    _check(len(sizes) >= 1, "KV cache tensor must have at least one dimension")
    if page_first:
        _check(sizes[0] > 0, "page dimension must be non-zero")
        num_pages, prefix = sizes[0], 1
        prefix_stride = 0
        page_stride = strides[0] * es
        suffix = dense_span(sizes, strides, 1) * es
        if num_pages > 1:
            _check(page_stride >= suffix, "KV cache pages overlap")
    else:
        _check(len(sizes) >= 2, "non-page-first KV cache tensor must have at least two dimensions")
        _check(sizes[0] > 0, "prefix dimension must be non-zero")
        _check(sizes[1] > 0, "page dimension must be non-zero")
        prefix, num_pages = sizes[0], sizes[1]
        prefix_stride = strides[0] * es
        page_stride = strides[1] * es
        suffix = dense_span(sizes, strides, 2) * es
        axes = []
        if prefix > 1:
            axes.append((prefix_stride, prefix))
        if num_pages > 1:
            axes.append((page_stride, num_pages))
        axes.sort()
        span = suffix
        for stride, size in axes:
            _check(stride >= span, "KV cache prefix/page regions overlap")
            span += (size - 1) * stride
    _check(page_stride > 0, "page_stride must be positive")
    return num_pages, prefix, page_stride, suffix, prefix_stride


def _jobs(layers, store, layer_names, offsets, byte_sizes, indices_flat, indices_offsets):
    n = len(layer_names)
    _check(len(offsets) == n, "offsets length mismatch")
    _check(len(byte_sizes) == n, "byte_sizes length mismatch")
    _check(len(indices_offsets) == n + 1, "indices_offsets size must be num_jobs + 1")
    if n == 0:
        return []
    _check(indices_offsets[0] >= 0, "indices_offsets[0] must be non-negative")
    _check(indices_offsets[-1] <= len(indices_flat), "indices_offsets.back() exceeds indices_flat.numel()")
    for i in range(n):
        _check(offsets[i] >= 0, f"negative store offset at job {i}")
        _check(byte_sizes[i] >= 0, f"negative byte size at job {i}")
        _check(indices_offsets[i] <= indices_offsets[i + 1], f"indices_offsets must be non-decreasing at job {i}")
        _check(offsets[i] <= store.size, f"store offset out of range at job {i}")
        _check(byte_sizes[i] <= store.size - offsets[i], f"store range out of bounds at job {i}")
    jobs = []
    for i, name in enumerate(layer_names):
        _check(name in layers, f"layer not registered: {name}")
        L = layers[name]
        num_pages, prefix, page_stride, suffix, prefix_stride = page_copy_shape(L.sizes, L.strides, L.es,
                                                                                L.page_first)
        ids = np.asarray(indices_flat[indices_offsets[i]:indices_offsets[i + 1]], np.int64)
        _check(byte_sizes[i] == prefix * len(ids) * suffix, f"byte_size mismatch at job {i}")
        jobs.append((L, offsets[i], ids, prefix, page_stride, suffix, prefix_stride))
    return jobs


def scatter_pages(layers, store, layer_names, offsets, byte_sizes, indices_flat, indices_offsets):
    """store -> layers: layer[p*prefix_stride + ids[i]*page_stride + o] =
    store[off + (p*n_sel + i)*suffix + o]; block id 0 skipped (kernels.cu:86-123)."""
    for L, off, ids, prefix, page_stride, suffix, prefix_stride in _jobs(
            layers, store, layer_names, offsets, byte_sizes, indices_flat, indices_offsets):
        for i, blk in enumerate(ids):
            if blk == 0:
                continue
            for p in range(prefix):
                s = off + (p * len(ids) + i) * suffix
                d = p * prefix_stride + int(blk) * page_stride
                L.mem[d:d + suffix] = store[s:s + suffix]


def gather_pages(layers, store, layer_names, offsets, byte_sizes, indices_flat, indices_offsets):
    """layers -> store, same mapping (kernels.cu:7-45); block id 0 skipped."""
    for L, off, ids, prefix, page_stride, suffix, prefix_stride in _jobs(
            layers, store, layer_names, offsets, byte_sizes, indices_flat, indices_offsets):
        for i, blk in enumerate(ids):
            if blk == 0:
                continue
            for p in range(prefix):
                s = off + (p * len(ids) + i) * suffix
                d = p * prefix_stride + int(blk) * page_stride
                store[s:s + suffix] = L.mem[d:d + suffix]
