"""Low-rank quantised proximity (use_qlora=True, quant_mode="int8") on the device.

* the proximity operator applied through leaf sums equals the dense finishprox'd matrix
  (the exact path, itself bit-exact with the oracle) times a block, to fp32 rounding;
* the tensor-core product and its fused top-k equal a numpy evaluation of the same
  quantised factors bit for bit (values and indices, ties by index);
* the factors approximate the exact proximity close to the best rank-k PSD approximation;
  RMSE and top-50 recall against the exact matrix are stated in the assertions.
"""
import numpy as np
import pytest

from _helpers import synth

pytestmark = pytest.mark.gpu

TOL_APPLY = 2e-5      # max |S X - dense S @ X| relative to max |S @ X| (fp32 sums)
RMSE_FACTOR = 1.25    # RMSE(A A^T - S) <= 1.25 x RMSE of the best rank-k PSD approximation + 1e-3


def _fit(X, y, qlora, rank=32, **kw):
    import rfx_b200
    n, p = X.shape
    est = rfx_b200.RandomForestClassifier(
        nsample=n, ntree=kw.pop("ntree", 40), mdim=p, mtry=kw.pop("mtry", 3),
        minndsize=kw.pop("minndsize", 1), compute_proximity=True, compute_importance=False,
        use_qlora=qlora, quant_mode="int8", rank=rank, **kw)
    est.fit(X, y)
    return est


def _topk_numpy(q, s, k, rows=None):
    """Top-k of P_ij = (dot(q_i, q_j) * s_i) * s_j in float32, j != i, value desc / index asc."""
    R = q.shape[0]
    acc = (q.astype(np.int64) @ q.astype(np.int64).T).astype(np.float32)
    P = (acc * s[:, None]) * s[None, :]
    rows = range(R) if rows is None else rows
    idx = np.full((len(rows), k), -1, np.int32)
    val = np.full((len(rows), k), -np.inf, np.float32)
    for a, i in enumerate(rows):
        cols = np.array([j for j in range(R) if j != i])
        v = P[i, cols]
        o = np.lexsort((cols, -v))[:k]
        idx[a, : len(o)] = cols[o]
        val[a, : len(o)] = v[o]
    return P, idx, val


def test_prox_apply_matches_dense_operator():
    import torch
    X, y = synth("class", 1200, 10, 11)
    dense = _fit(X, y, qlora=False).get_proximity_matrix().astype(np.float64)
    est = _fit(X, y, qlora=True)
    R = dense.shape[0]
    rng = np.random.default_rng(5)
    Z = rng.normal(size=(R, 24)).astype(np.float32)
    dev = torch.device("cuda", 0)
    Zt = torch.from_numpy(Z).to(dev)
    Yt = torch.empty_like(Zt)
    torch.cuda.synchronize()
    est._context().prox_apply(Zt.data_ptr(), Z.shape[1], Yt.data_ptr())
    got = Yt.cpu().numpy().astype(np.float64)
    want = dense @ Z.astype(np.float64)
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err < TOL_APPLY, err


def test_product_and_topk_bit_exact_vs_numpy():
    X, y = synth("multiclass", 1000, 12, 12)  # R = 1000: 8 row blocks, 4 column tiles
    est = _fit(X, y, qlora=True, rank=48)
    q, s = est.get_lowrank_quantized()
    assert q.shape == (1000, 48) and s.shape == (1000,)
    k = 50
    P, idx_np, val_np = _topk_numpy(q, s, k)
    got = est.get_lowrank_product()
    assert np.array_equal(got.view(np.uint32), P.view(np.uint32))
    idx, val = est.get_lowrank_topk(k)
    assert np.array_equal(val.view(np.uint32), val_np.view(np.uint32))
    assert np.array_equal(idx, idx_np)
    # a row range that does not start on a tile boundary
    idx2, val2 = est.get_lowrank_topk(7, 333, 777)
    _, i7, v7 = _topk_numpy(q, s, 7, rows=range(333, 777))
    assert np.array_equal(idx2, i7) and np.array_equal(val2.view(np.uint32), v7.view(np.uint32))
    A, B, r = est.get_lowrank_factors()
    assert r == 48 and A.dtype == np.float64 and np.array_equal(A, B)
    assert np.array_equal(A.astype(np.float32), (s[:, None] * q.astype(np.float32)))


def test_topk_fewer_rows_than_k():
    X, y = synth("class", 40, 6, 13)
    est = _fit(X, y, qlora=True, rank=8, ntree=10)
    q, s = est.get_lowrank_quantized()
    idx, val = est.get_lowrank_topk(50)
    _, idx_np, val_np = _topk_numpy(q, s, 50)
    assert np.array_equal(idx, idx_np)
    assert (idx[:, 39:] == -1).all() and np.isneginf(val[:, 39:]).all()
    assert np.array_equal(val.view(np.uint32), val_np.view(np.uint32))


def test_factor_quality_vs_exact_proximity():
    X, y = synth("multiclass", 1500, 10, 14)
    rank = 64
    S = _fit(X, y, qlora=False, ntree=60).get_proximity_matrix().astype(np.float64)
    est = _fit(X, y, qlora=True, rank=rank, ntree=60)
    A, _, _ = est.get_lowrank_factors()
    approx = A @ A.T
    rmse = np.sqrt(np.mean((approx - S) ** 2))
    w, V = np.linalg.eigh(S)
    top = np.argsort(w)[::-1][:rank]
    wk = np.clip(w[top], 0, None)
    best = (V[:, top] * wk) @ V[:, top].T
    rmse_best = np.sqrt(np.mean((best - S) ** 2))
    assert rmse <= RMSE_FACTOR * rmse_best + 1e-3, (rmse, rmse_best)
    # top-50 recall against the exact matrix (stated, loose bar)
    idx, _ = est.get_lowrank_topk(50)
    Sx = S.copy()
    np.fill_diagonal(Sx, -np.inf)
    exact = np.argsort(-Sx, axis=1, kind="stable")[:, :50]
    recall = np.mean([len(np.intersect1d(idx[i], exact[i])) / 50 for i in range(S.shape[0])])
    print(f"low-rank rank={rank}: rmse={rmse:.4g} best={rmse_best:.4g} top50 recall={recall:.3f}")
    assert recall > 0.3, recall


def _topk_ref(q, s, k):
    """Exact top-k of the quantised product for every row (numpy, float32 like the kernel)."""
    acc = (q.astype(np.int64) @ q.astype(np.int64).T).astype(np.float32)
    P = (acc * s[:, None]) * s[None, :]
    R = P.shape[0]
    Pm = P.copy()
    np.fill_diagonal(Pm, -np.inf)
    order = np.argsort(-Pm, axis=1, kind="stable")[:, :k]  # value desc, index asc
    val = np.take_along_axis(Pm, order, axis=1)
    idx = order.astype(np.int32)
    idx[np.isneginf(val)] = -1
    return P, idx, val.astype(np.float32)


@pytest.mark.parametrize("k", [1, 50, 64])
def test_topk_kernel_adversarial_factors(k):
    """Caller-supplied factors with duplicated rows (ties broken by index), zero rows, zero
    scales and negative products, over 20 column tiles (the early stop engages)."""
    import rfx_b200
    rng = np.random.default_rng(21)
    R, rank = 5000, 37
    q = rng.integers(-127, 128, size=(R, rank)).astype(np.int8)
    q[rng.integers(0, R, 600)] = q[rng.integers(0, R, 600)]  # duplicate rows -> equal values
    q[10:20] = 0                                              # zero rows
    s = rng.uniform(0.001, 0.02, size=R).astype(np.float32)
    s[rng.integers(0, R, 200)] = np.float32(0.01)            # shared scales -> more ties
    s[30:35] = 0.0                                            # zero scales
    ctx = rfx_b200.Context(0)
    ctx.lowrank_set_factors(q, s)
    P, idx_np, val_np = _topk_ref(q, s, k)
    idx, val = ctx.lowrank_topk(k, 0, R)
    assert np.array_equal(idx, idx_np)
    assert np.array_equal(val.view(np.uint32), val_np.view(np.uint32))
    # an interleaved row range
    idx2, val2 = ctx.lowrank_topk(k, 1234, 3456)
    assert np.array_equal(idx2, idx_np[1234:3456])
    assert np.array_equal(val2.view(np.uint32), val_np[1234:3456].view(np.uint32))
    dense = ctx.lowrank_product(100, 300, R)
    assert np.array_equal(dense.view(np.uint32), P[100:300].view(np.uint32))
    # shares of the kernel's row order (how a sharded fit splits the rows over GPUs)
    seen = []
    for part in range(3):
        rows, ip, vp = ctx.lowrank_topk_part(k, part, 3)
        assert np.array_equal(ip, idx_np[rows])
        assert np.array_equal(vp.view(np.uint32), val_np[rows].view(np.uint32))
        seen.append(rows)
    assert np.array_equal(np.sort(np.concatenate(seen)), np.arange(R))
