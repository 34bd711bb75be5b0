"""CPU restatement of the reference's leaf-assignment queries (test infrastructure only).

Follows include/rf_random_forest.hpp:296-365 and src/rf_random_forest.cpp:1543-1610 (leaf
assignments), 3724-3770 (find_terminal_node), 4110-4277 (outlier scores), 4605-4787 (leaf
proximity, top-k similar), 4789-4850 (predict_leaf_assignments) and
python/randomforest_py.cpp:2496-2560 (predict_top_k_similar).  Pure Python / numpy for
small cases.  The rankings the reference leaves to libstdc++'s std::partial_sort are
restated with that algorithm (heap select, then heap sort) so tied rows come out in the
reference's order.
"""
import numpy as np


def _walk(nodestatus, bestvar, xbestsplit, treemap, x, maxnode, mdim, cat=None):
    """Terminal node of one row (find_terminal_node, numeric features; predict_leaf's
    categorical rule: jcat = (int)(x + 0.5) in [0, cat) goes right, otherwise no move)."""
    node = 0
    for _ in range(maxnode):
        if nodestatus[node] == -1:
            break
        m = int(bestvar[node])
        if not (0 <= m < mdim):
            break
        v = np.float32(x[m])
        if cat is None or cat[m] == 1:
            nxt = treemap[2 * node] if v <= xbestsplit[node] else treemap[2 * node + 1]
        else:
            y = np.float32(v + np.float32(0.5))
            jcat = int(y) if (y >= -2147483648.0 and y < 2147483648.0) else -2147483648
            if not (0 <= jcat < cat[m]):
                break
            nxt = treemap[2 * node + 1]
        node = int(nxt)
    return node


def leaf_assignments(trees, X):
    """int16 [ntree][N] for the grown rows X [N][p] (src/rf_random_forest.cpp:1551-1610)."""
    T, M = trees["nodestatus"].shape
    N, p = X.shape
    out = np.zeros((T, N), np.int16)
    for t in range(T):
        st, bv, xb, tm = (trees["nodestatus"][t], trees["bestvar"][t], trees["xbestsplit"][t],
                          trees["treemap"][t])
        for n in range(N):
            out[t, n] = np.int16(_walk(st, bv, xb, tm, X[n], M, p))
    return out


def predict_leaf_assignments(trees, Xn, cat):
    """int16 [n][ntree] (src/rf_random_forest.cpp:4789-4850)."""
    T, M = trees["nodestatus"].shape
    n, p = Xn.shape
    out = np.zeros((n, T), np.int16)
    for t in range(T):
        st, bv, xb, tm = (trees["nodestatus"][t], trees["bestvar"][t], trees["xbestsplit"][t],
                          trees["treemap"][t])
        for s in range(n):
            out[s, t] = np.int16(_walk(st, bv, xb, tm, Xn[s], M, p, cat))
    return out


# ---- libstdc++ std::partial_sort (heap select + heap sort) ---------------------------------
def _adjust_heap(a, first, hole, length, value, comp):
    top = hole
    child = hole
    while child < (length - 1) // 2:
        child = 2 * (child + 1)
        if comp(a[first + child], a[first + child - 1]):
            child -= 1
        a[first + hole] = a[first + child]
        hole = child
    if (length & 1) == 0 and child == (length - 2) // 2:
        child = 2 * (child + 1)
        a[first + hole] = a[first + child - 1]
        hole = child - 1
    parent = (hole - 1) // 2
    while hole > top and comp(a[first + parent], value):
        a[first + hole] = a[first + parent]
        hole = parent
        parent = (hole - 1) // 2
    a[first + hole] = value


def _make_heap(a, first, last, comp):
    length = last - first
    if length < 2:
        return
    parent = (length - 2) // 2
    while True:
        _adjust_heap(a, first, parent, length, a[first + parent], comp)
        if parent == 0:
            return
        parent -= 1


def _pop_heap(a, first, last, result, comp):
    value = a[result]
    a[result] = a[first]
    _adjust_heap(a, first, 0, last - first, value, comp)


def partial_sort(a, k, comp):
    """std::partial_sort(a.begin(), a.begin() + k, a.end(), comp) on a Python list."""
    first, middle, last = 0, k, len(a)
    _make_heap(a, first, middle, comp)
    for i in range(middle, last):
        if comp(a[i], a[first]):
            _pop_heap(a, first, middle, i, comp)
    while middle - first > 1:
        middle -= 1
        _pop_heap(a, first, middle, middle, comp)
    return a


def top_k_similar(leaves, oob, q, k=10, exclude_self=True):
    """(indices, similarities) of get_top_k_similar (src/rf_random_forest.cpp:4677-4787);
    oob [ntree][N] bool.  Empty when the query was never OOB or nothing matches."""
    T, N = leaves.shape
    trees = [t for t in range(T) if oob[t, q]]
    if not trees:
        return np.zeros(0, np.int32), np.zeros(0, np.float32)
    cnt = np.zeros(N, np.int64)
    for t in trees:
        same = leaves[t] == leaves[t, q]
        if exclude_self:
            same[q] = False
        cnt += same
    norm = np.float32(1.0) / np.float32(len(trees))
    ic = [(i, int(cnt[i])) for i in range(N) if not (exclude_self and i == q) and cnt[i] > 0]
    kk = min(k, len(ic))
    if kk > 0:
        partial_sort(ic, kk, lambda a, b: a[1] > b[1])
    idx = np.array([ic[e][0] for e in range(kk)], np.int32)
    sim = np.array([np.float32(ic[e][1]) * norm for e in range(kk)], np.float32)
    return idx, sim


def predict_top_k_similar(train_leaves, new_leaves, k):
    """(indices [n][k], similarities [n][k]) over all trees (python/randomforest_py.cpp:2496-2560)."""
    T, N = train_leaves.shape
    n = new_leaves.shape[0]
    idx = np.zeros((n, k), np.int32)
    sim = np.zeros((n, k), np.float32)
    for q in range(n):
        s = np.zeros(N, np.float32)
        for t in range(T):
            s += (train_leaves[t] == new_leaves[q, t]).astype(np.float32)
        s = (s / np.float32(T)).astype(np.float32)
        order = list(range(N))
        partial_sort(order, k, lambda a, b: s[a] > s[b])
        idx[q] = order[:k]
        sim[q] = s[order[:k]]
    return idx, sim


def leaf_proximity(leaves, oob, i, j):
    """compute_proximity_from_leaves (src/rf_random_forest.cpp:4605-4642)."""
    trees = [t for t in range(leaves.shape[0]) if oob[t, i]]
    if not trees:
        return np.float32(0.0)
    m = sum(1 for t in trees if leaves[t, i] == leaves[t, j])
    return np.float32(m) / np.float32(len(trees))


def outlier_stats(raw, labels=None):
    """{class (or -1): (median, MAD)} of the raw measures (:4201-4272)."""
    stats = {}
    keys = np.unique(labels) if labels is not None else [-1]
    for c in keys:
        v = raw[labels == c] if labels is not None else raw
        med = np.sort(v)[len(v) // 2]
        dev = np.sort(np.abs((v - med).astype(np.float32)))
        mad = dev[len(v) // 2]
        if mad < np.float32(1e-10):
            mad = np.float32(1.0)
        stats[int(c)] = (np.float32(med), np.float32(mad))
    return stats


def _normalise(raw, labels):
    """(raw - median) / MAD, per class when labels are given (:4201-4272)."""
    out = np.zeros_like(raw)
    stats = outlier_stats(raw, labels)
    for c, (med, mad) in stats.items():
        g = np.nonzero(labels == c)[0] if labels is not None else np.arange(raw.shape[0])
        out[g] = ((raw[g] - med).astype(np.float32) / mad).astype(np.float32)
    return out


def predict_outlier_scores(train_leaves, new_leaves, stats, greedy, n_anchors, classes=None):
    """RandomForest::predict_outlier_scores (src/rf_random_forest.cpp:5210-5330): per new row
    the proximity (shared trees / ntree, over all trees) to every training row; raw = count /
    sum of squares over the positive ones (greedy: the n_anchors largest, in descending order;
    full: all of them in row order), normalised with the training statistics (per predicted
    class for a classifier)."""
    T, N = train_leaves.shape
    out = np.zeros(new_leaves.shape[0], np.float32)
    for s in range(new_leaves.shape[0]):
        cnt = np.zeros(N, np.int64)
        for t in range(T):
            cnt += train_leaves[t] == new_leaves[s, t]
        prox = (cnt.astype(np.float32) / np.float32(T)).astype(np.float32)
        pos = prox[prox > 0]
        if greedy and n_anchors > 0:
            pos = np.sort(pos)[::-1][:n_anchors]
        ss = np.float32(0.0)
        for v in pos:
            ss = np.float32(ss + np.float32(v * v))
        n = len(pos)
        raw = (np.float32(n) / ss if (ss > np.float32(1e-10) and n > 0)
               else np.float32(N) * np.float32(1e10))
        key = int(classes[s]) if classes is not None else -1
        med, mad = stats.get(key, (np.float32(0.0), np.float32(1.0)))
        out[s] = np.float32(np.float32(raw - med) / mad)
    return out


def outlier_raw_greedy(leaves, anchors, n_anchors):
    """Greedy raw measure in the reference's float32 order (:4127-4160)."""
    T, N = leaves.shape
    raw = np.zeros(N, np.float32)
    for n in range(N):
        s = np.float32(0.0)
        for a in anchors:
            if a == n:
                continue
            shared = int(np.count_nonzero(leaves[:, n] == leaves[:, a]))
            prox = np.float32(shared) / np.float32(T)
            s = np.float32(s + np.float32(prox * prox))
        raw[n] = (np.float32(n_anchors) / s if s > np.float32(1e-10)
                  else np.float32(n_anchors) * np.float32(1e10))
    return raw


def outlier_raw_full(leaves):
    """Full raw measure: (N - 1) / sum over other rows of (shared trees / T)^2, the sum formed
    exactly and rounded once (the reference adds float terms in hash-map order)."""
    T, N = leaves.shape
    raw = np.zeros(N, np.float32)
    for n in range(N):
        c = np.zeros(N, np.int64)
        for t in range(T):
            c += leaves[t] == leaves[t, n]
        c[n] = 0
        pss = np.float32(float(np.sum(c * c)) / (float(T) * float(T)))
        raw[n] = (np.float32(N - 1) / pss if pss > np.float32(1e-10)
                  else np.float32(N) * np.float32(1e10))
    return raw


def outlier_scores(raw, labels=None):
    return _normalise(raw.astype(np.float32), labels)
