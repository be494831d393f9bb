"""The input upload ring (``tx.Prefetcher``, C ABI ``tx_prefetch_*``).

Batches queued through the ring arrive intact and in order; a buffer is not
refilled while compute work issued before a later ``get`` still has to read
it (the copy stream runs beside the compute stream, so this is the ordering
the ring must keep); putting further ahead than the ring holds is refused; and
a model fed from the ring gives the same outputs as one fed through
``tx.Tensor``.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _batches(n, rows=64, cols=33, seed=3):
    rng = np.random.default_rng(seed)
    import tynx_b200 as tx

    return [(tx.pinned(rng.standard_normal((rows, cols)).astype(np.float32)),
             tx.pinned(rng.integers(0, 10, rows).astype(np.int64))) for _ in range(n)]


def test_batches_arrive_intact_and_in_order():
    import tynx_b200 as tx

    host = _batches(6)
    pf = tx.Prefetcher(*host[0], depth=3)
    pf.put(*host[0])
    pf.put(*host[1])
    for i in range(6):
        tx_x, tx_y = pf.get()
        if i + 2 < 6:
            pf.put(*host[i + 2])
        np.testing.assert_array_equal(tx_x.numpy(), host[i][0])
        np.testing.assert_array_equal(tx_y.numpy(), host[i][1])
    pf.close()


def test_buffer_refill_waits_for_earlier_readers():
    import tynx_b200 as tx

    host = _batches(4, rows=256, cols=256)
    pf = tx.Prefetcher(*host[0], depth=2)
    a = tx.randn(4096, 4096)
    pf.put(*host[0])
    x0, _ = pf.get()
    # a long product ahead of the read of batch 0 on the compute stream
    slow = tx.matmul(a, a)
    slow = tx.matmul(slow, a)
    s0 = (x0 * 1.0).sum()  # reads buffer 0 after the products
    pf.put(*host[1])
    pf.get()               # releases buffer 0: everything above was issued before it
    pf.put(*host[2])       # refills buffer 0: must wait for the read above
    want = float(host[0][0].astype(np.float64).sum())
    got = float(s0.item())
    assert abs(got - want) <= 1e-3 * max(1.0, abs(want)), (got, want)
    assert np.isfinite(float(slow.sum().item()))
    pf.close()


def test_depth_three_refill_waits_for_readers_issued_before_the_next_get():
    """With depth 3, batch g is valid for work issued before get g + 1 while
    two more batches upload; put g + 3 refills its buffer only after that work."""
    import tynx_b200 as tx

    host = _batches(5, rows=256, cols=256)
    pf = tx.Prefetcher(*host[0], depth=3)
    a = tx.randn(4096, 4096)
    pf.put(*host[0])
    pf.put(*host[1])
    pf.put(*host[2])
    x0, _ = pf.get()
    slow = tx.matmul(tx.matmul(a, a), a)
    s0 = (x0 * 1.0).sum()  # reads buffer 0 behind the products, before the next get
    x1, _ = pf.get()       # releases buffer 0 for put 3
    pf.put(*host[3])       # refills buffer 0: must wait for the read above
    s1 = (x1 * 1.0).sum()
    x2, _ = pf.get()
    pf.put(*host[4])       # refills buffer 1 after the read of x1
    x3, _ = pf.get()
    for got, want in ((s0, host[0][0]), (s1, host[1][0])):
        want = float(want.astype(np.float64).sum())
        assert abs(float(got.item()) - want) <= 1e-3 * max(1.0, abs(want)), (float(got.item()), want)
    np.testing.assert_array_equal(x2.numpy(), host[2][0])
    np.testing.assert_array_equal(x3.numpy(), host[3][0])
    assert np.isfinite(float(slow.sum().item()))
    pf.close()


def test_put_refuses_to_run_past_the_ring():
    import tynx_b200 as tx

    host = _batches(3)
    pf = tx.Prefetcher(*host[0], depth=2)
    pf.put(*host[0])
    pf.put(*host[1])
    with pytest.raises(Exception):
        pf.put(*host[2])  # both buffers hold batches nobody has taken
    pf.get()
    with pytest.raises(Exception):
        pf.put(*host[2])  # buffer 0's batch is taken but not yet released by a later get
    pf.get()
    pf.put(*host[2])
    x, y = pf.get()
    np.testing.assert_array_equal(x.numpy(), host[2][0])
    pf.close()


def test_model_outputs_match_plain_tensors():
    import tynx_b200 as tx
    from tynx_b200 import workloads

    wl = workloads.mlp_classifier(batch=128)
    model = tx.load(wl.onnx, trainable="auto")
    host = []
    for step in range(4):
        b = wl.make_batch(step)
        host.append((tx.pinned(b["x"].astype(np.float32)), tx.pinned(b["y"].astype(np.int64))))
    pf = tx.Prefetcher(*host[0], depth=3)
    pf.put(*host[0])
    pf.put(*host[1])
    for i in range(4):
        x, _ = pf.get()
        out = model(x).numpy()
        if i + 2 < 4:
            pf.put(*host[i + 2])
        ref = model(tx.Tensor(host[i][0])).numpy()
        np.testing.assert_array_equal(out, ref)
    pf.close()


def test_put_rejects_mismatched_batches():
    import tynx_b200 as tx

    host = _batches(1)
    pf = tx.Prefetcher(*host[0], depth=2)
    with pytest.raises(TypeError):
        pf.put(host[0][0].astype(np.float64), host[0][1])
    with pytest.raises(ValueError):
        pf.put(host[0][0])
    pf.close()
