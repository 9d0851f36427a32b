"""Host logic of the host-input pipeline: the pieces a call copies and runs."""

import pytest

from kvblockmass_b200 import _lib
from kvblockmass_b200.ops import _host_pieces

P1, P2 = _lib.KVBM_STAGE_PASS1, _lib.KVBM_STAGE_PASS2


@pytest.mark.parametrize("U,G,N,by_rows", [(8, 4, 32768, True), (8, 4, 32768, False), (3, 1, 9000, True),
                                            (2, 4, 4096, True), (2, 4, 4095, True), (1, 8, 131072, True),
                                            (4, 1, 700, False), (1, 2, 5000, True)])
def test_pieces_cover_every_head_and_row_once(U, G, N, by_rows):
    pieces = _host_pieces(U, G, N, by_rows)
    rowed = by_rows and N >= 4096  # row pieces only where asked for and long enough
    # unit 0 first, in pass-1 pieces; with row pieces the last unit comes last,
    # cut the same way; every other unit is one piece with both passes
    split = {0} | ({U - 1} if rowed else set())
    order = [pc[0] for pc in pieces]
    assert order == sorted(order)
    for u in range(U):
        mine = [pc for pc in pieces if pc[0] == u]
        if u not in split:
            assert len(mine) == 1
            pc = mine[0]
            assert pc[3] == P1 | P2 and pc[1] == (0, G) and pc[2] is None and pc[4]
            continue
        assert all(pc[3] == P1 for pc in mine)
        # k travels with the unit's first piece only
        assert [pc[4] for pc in mine] == [True] + [False] * (len(mine) - 1)
        # every (head, row) of the unit exactly once
        cover = {}
        for _, (h0, h1), rows, _, _ in mine:
            r0, r1 = rows if rows is not None else (0, N)
            assert 0 <= r0 < r1 <= N and r0 % 128 == 0 and (r1 % 128 == 0 or r1 == N)
            for h in range(h0, h1):
                cover.setdefault(h, []).append((r0, r1))
        assert sorted(cover) == list(range(G))
        for h, rr in cover.items():
            rr.sort()
            assert rr[0][0] == 0 and rr[-1][1] == N
            assert all(a[1] == b[0] for a, b in zip(rr, rr[1:]))
        assert any(pc[2] is not None for pc in mine) == rowed
        if rowed:  # the last rows come first
            assert 2 <= len(mine) <= 8
            assert [pc[2] for pc in mine] == sorted((pc[2] for pc in mine), reverse=True)
