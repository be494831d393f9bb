"""Host-side arithmetic of the eager operations, checked without a GPU:
the strided-view plan behind basic indexing (`Tensor.__getitem__`) against
numpy's basic indexing, and the pooled output length of `max_pool2d` /
`avg_pool2d` against the oracle's (torch / ONNX ceil-mode rule: a window may
not start in the right padding)."""

import numpy as np
import pytest

from oracle.flex_oracle import _pool_axis
from tynx_b200._core import _index_plan
from tynx_b200.nn.functional import _pool_out


def _gather(base: np.ndarray, plan) -> np.ndarray:
    """The elements the plan addresses, by explicit element indices (every
    index is checked to lie inside the base tensor)."""
    offset, shape, strides, out_shape = plan
    flat = base.reshape(-1)
    idx = np.full(shape, offset, dtype=np.int64)
    for axis, (n, st) in enumerate(zip(shape, strides)):
        view = [1] * len(shape)
        view[axis] = n
        idx = idx + (np.arange(n, dtype=np.int64) * st).reshape(view)
    if idx.size:
        assert idx.min() >= 0 and idx.max() < flat.size
    return flat[idx].reshape(out_shape)


def _random_index(rng, ndim):
    parts = []
    n_real = int(rng.integers(0, ndim + 1))
    for _ in range(n_real):
        kind = rng.integers(0, 3)
        if kind == 0:
            parts.append(int(rng.integers(-3, 3)))
        else:
            start = None if rng.random() < 0.3 else int(rng.integers(-8, 8))
            stop = None if rng.random() < 0.3 else int(rng.integers(-8, 8))
            step = None if rng.random() < 0.3 else int(rng.choice([-3, -2, -1, 1, 2, 3]))
            parts.append(slice(start, stop, step))
    for _ in range(int(rng.integers(0, 2))):
        parts.insert(int(rng.integers(0, len(parts) + 1)), None)
    if rng.random() < 0.5:
        parts.insert(int(rng.integers(0, len(parts) + 1)), Ellipsis)
    return tuple(parts)


def test_index_plan_matches_numpy_basic_indexing():
    rng = np.random.default_rng(0)
    checked = 0
    for _ in range(3000):
        ndim = int(rng.integers(1, 5))
        shape = tuple(int(s) for s in rng.integers(1, 6, ndim))
        base = np.arange(int(np.prod(shape)), dtype=np.float32).reshape(shape)
        index = _random_index(rng, ndim)
        try:
            want = base[index]
        except IndexError:
            with pytest.raises(IndexError):
                _index_plan(shape, index)
            continue
        got = _gather(base, _index_plan(shape, index))
        assert got.shape == want.shape, (shape, index)
        np.testing.assert_array_equal(got, want)
        checked += 1
    assert checked > 2000


def test_index_plan_rejects_advanced_and_invalid_indices():
    with pytest.raises(NotImplementedError):
        _index_plan((4, 5), ([0, 1],))
    with pytest.raises(IndexError):
        _index_plan((4, 5), (0, 0, 0))
    with pytest.raises(IndexError):
        _index_plan((4, 5), (Ellipsis, Ellipsis))
    with pytest.raises(IndexError):
        _index_plan((4, 5), (4,))
    with pytest.raises(TypeError):
        _index_plan((4, 5), (1.5,))


@pytest.mark.parametrize("ceil", [False, True])
def test_pool_output_length_matches_oracle(ceil):
    for size in range(1, 24):
        for k in range(1, 6):
            for s in range(1, 4):
                for p in range(0, k // 2 + 1):
                    for d in (1, 2):
                        eff = d * (k - 1) + 1
                        if size + 2 * p < eff:
                            with pytest.raises(ValueError):
                                _pool_out(size, k, s, p, d, ceil)
                            continue
                        _, want = _pool_axis(size, k, s, d, p, p, "NOTSET", ceil)
                        assert _pool_out(size, k, s, p, d, ceil) == want, (size, k, s, p, d, ceil)


def test_repeat_plan_matches_numpy_tile():
    from tynx_b200._core import _repeat_plan

    rng = np.random.default_rng(1)
    for _ in range(500):
        ndim = int(rng.integers(0, 4))
        shape = tuple(int(s) for s in rng.integers(1, 5, ndim))
        sizes = tuple(int(r) for r in rng.integers(0, 4, ndim + int(rng.integers(0, 3))))
        if not sizes:
            continue
        x = rng.standard_normal(shape).astype(np.float32)
        inter, tiled, final = _repeat_plan(shape, sizes)
        got = np.broadcast_to(x.reshape(inter), tiled).reshape(final)
        np.testing.assert_array_equal(got, np.tile(x, sizes))
    with pytest.raises(ValueError):
        _repeat_plan((2, 3), (2,))
    with pytest.raises(ValueError):
        _repeat_plan((2,), (-1,))
