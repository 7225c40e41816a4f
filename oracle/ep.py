"""Expert-parallel dispatch / combine semantics (test infrastructure only).

The reference drives MoRI's EpDispatchCombineOp (a third-party package, `mori`,
absent from the reference tree; version not recorded there) through
aiter/dist/device_communicators/all2all.py:21-98 and
op_tests/multigpu_tests/test_dispatch_combine.py:76-171.  What that test fixes:
rank r owns experts [r*E/W, (r+1)*E/W); dispatch sends each token, with its
weights, scales and top-k ids, to every rank owning one of its experts and returns
the received rows and their count; the EP MoE runs on them with the rank's expert
mask; combine returns, per source token, the sum over ranks of those outputs (the
test's `run_ref`, :17-62, sums the per-rank masked MoE outputs).  MoRI's order of
received rows is not fixed by the test (it compares after combine); aiter_b200's
is: source 0's tokens, then source 1's, ..., each in token order.  Combine sums
the destinations in rank order in fp32 and rounds once (MoRI's accumulation is
not visible to the test, whose tolerance covers either).
"""
import numpy as np


def destinations(ids, experts_per_rank, world):
    """Sorted ranks owning at least one of a token's experts (ids outside
    [0, world * experts_per_rank) go nowhere)."""
    ids = np.asarray(ids).reshape(-1)
    ids = ids[(ids >= 0) & (ids < experts_per_rank * world)]
    return sorted(set((ids // experts_per_rank).tolist()))


def dispatch(per_rank, experts_per_rank, world):
    """per_rank: list of dicts with 'tokens' [T, H], 'weights' [T, k], 'ids' [T, k]
    and optionally 'scales' [T, S].  Returns per destination a dict of the received
    arrays in receive order plus 'src' (source, token) pairs."""
    out = []
    for d in range(world):
        rows = {"tokens": [], "weights": [], "ids": [], "scales": [], "src": []}
        for s, inp in enumerate(per_rank):
            for t in range(inp["ids"].shape[0]):
                if d in destinations(inp["ids"][t], experts_per_rank, world):
                    rows["tokens"].append(inp["tokens"][t])
                    rows["weights"].append(inp["weights"][t])
                    rows["ids"].append(inp["ids"][t])
                    if "scales" in inp:
                        rows["scales"].append(inp["scales"][t])
                    rows["src"].append((s, t))
        out.append(rows)
    return out


def combine(outputs, received, per_rank_tokens, out_dtype_round):
    """outputs[d]: [recv_d, H] float array of rank d's results in receive order;
    received: dispatch()'s result.  Returns per source s: [T_s, H], the fp32 sum of
    its tokens' rows over the ranks they went to, in rank order, rounded once with
    out_dtype_round."""
    world = len(outputs)
    hidden = outputs[0].shape[1] if len(outputs[0]) else None
    res = []
    for s in range(world):
        T = per_rank_tokens[s]
        h = hidden if hidden is not None else next((o.shape[1] for o in outputs if len(o)), 0)
        acc = np.zeros((T, h), dtype=np.float32)
        for d in range(world):
            for i, (src, t) in enumerate(received[d]["src"]):
                if src == s:
                    acc[t] += np.asarray(outputs[d][i], dtype=np.float32)
        res.append(out_dtype_round(acc))
    return res
