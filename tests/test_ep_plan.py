"""EP peer-exchange offset plan (host arithmetic, no GPU): the dispatch segments of all
sources tile every owner's receive buffer exactly, the combine segments tile every
source's buffer exactly, and rows land where the NCCL all-to-all would put them."""

import numpy as np

from pluggy_b200.comm.ep_fused import EPComm


class _Stub(EPComm):
    def __init__(self, n, rank, E):  # no buffers: only plan()
        self.n, self.rank, self.E, self.el = n, rank, E, E // n


def _simulate(n, E, seed):
    rng = np.random.default_rng(seed)
    C = rng.integers(0, 5, size=(n, E))
    C[rng.integers(0, n), :] = 0  # a rank that routes nothing
    plans = [_Stub(n, r, E).plan(C) for r in range(n)]
    # every source's rows, labelled (src, expert, k) in its destination-then-expert order
    rows = {s: [(s, e, k) for e in range(E) for k in range(C[s, e])] for s in range(n)}
    recv = {r: [None] * plans[r]["R"] for r in range(n)}
    for s in range(n):
        pl = plans[s]
        for d in range(n):
            for k in range(pl["send"][d]):
                slot = pl["to_owner_off"][d] + k
                assert recv[d][slot] is None
                recv[d][slot] = rows[s][pl["start"][d] + k]
    for r in range(n):
        assert None not in recv[r]
        el = E // n
        # what an all-to-all would deliver: source-major, each block in expert order
        want = [x for s in range(n) for x in rows[s] if r * el <= x[1] < (r + 1) * el]
        assert recv[r] == want
        # the local expert ids the FFN is given
        lc = plans[r]["local_counts"].reshape(-1)
        ids = np.repeat(np.tile(np.arange(el), n), lc)
        assert [x[1] - r * el for x in recv[r]] == ids.tolist()
    back = {s: [None] * plans[s]["P"] for s in range(n)}
    for r in range(n):
        pl = plans[r]
        for s in range(n):
            for k in range(pl["recv"][s]):
                slot = pl["back_off"][s] + k
                assert back[s][slot] is None
                back[s][slot] = recv[r][pl["recv_off"][s] + k]
    for s in range(n):
        assert back[s] == rows[s]  # each row returns to its own position
    return plans


def test_plan_tiles_buffers_both_ways():
    for n, E, seed in [(2, 8, 0), (4, 16, 1), (8, 128, 2), (3, 6, 3)]:
        plans = _simulate(n, E, seed)
        assert all(p["R_max"] == plans[0]["R_max"] for p in plans)  # collective sizing agrees
