"""TEST INFRASTRUCTURE ONLY: how far the reference built with its stock CMake flags
(-O3 -mavx2 -mfma, GCC free to contract a*b+c into FMAs) departs from the un-fused build
(-ffp-contract=off) that the oracle, the golden fixtures and the device path follow.

    make -C oracle ref ref-stock REF=<reference tree>
    python oracle/stock_compare.py [ntree]

Fits config[1]'s data (seeded as bench.py) with both builds and prints
per-tree agreement of the tree arrays and of the forest-level results.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import oracle  # noqa: E402
from bench import CFG, calc_maxnode, make_data  # noqa: E402


def main(ntree=8):
    X, y = make_data(CFG["n"], CFG["p"])
    M = calc_maxnode(CFG["n"], CFG["minndsize"])
    kw = dict(ntree=ntree, mtry=CFG["mtry"], minndsize=CFG["minndsize"], maxnode=M)
    a = oracle.ref_fit(1, X, y, **kw)
    b = oracle.ref_fit(1, X, y, stock=True, **kw)
    keys = ("nodestatus", "bestvar", "xbestsplit", "treemap", "nodepred", "nnode")
    same = [all(np.array_equal(np.asarray(a[k][t]).view(np.uint8), np.asarray(b[k][t]).view(np.uint8))
                for k in keys) for t in range(ntree)]
    # first node where each differing tree departs (BFS order = the reference's visiting order)
    first = []
    for t in range(ntree):
        if same[t]:
            continue
        d = np.flatnonzero((a["bestvar"][t] != b["bestvar"][t]) |
                           (a["xbestsplit"][t].view(np.uint32) != b["xbestsplit"][t].view(np.uint32)) |
                           (a["nodepred"][t].view(np.uint32) != b["nodepred"][t].view(np.uint32)))
        first.append((t, int(d[0]) if len(d) else -1, int(a["nnode"][t]), int(b["nnode"][t])))
    oob = np.mean(a["oob_pred"].view(np.uint32) != b["oob_pred"].view(np.uint32))
    imp = np.mean(a["avimp"].view(np.uint32) != b["avimp"].view(np.uint32))
    print(f"config[1], {ntree} trees: {sum(same)} identical, {ntree - sum(same)} differ "
          f"(tree, first differing node, nnode un-fused, nnode stock): {first}")
    print(f"  OOB predictions differing: {100 * oob:.2f}% of rows; importance entries "
          f"differing: {100 * imp:.1f}%; OOB error un-fused {a['oob_error']:.6f} stock "
          f"{b['oob_error']:.6f}")


if __name__ == "__main__":
    main(int(sys.argv[1]) if len(sys.argv) > 1 else 8)
