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
    seen_k = set()
    cover = {}
    for u, (h0, h1), rows, stages, with_k in pieces:
        assert 0 <= u < U and 0 <= h0 < h1 <= G
        # k travels with the first piece of its unit, and only then
        assert with_k == (u not in seen_k)
        seen_k.add(u)
        r0, r1 = rows if rows is not None else (0, N)
        assert 0 <= r0 < r1 <= N and r0 % 128 == 0 and (r1 % 128 == 0 or r1 == N)
        for h in range(h0, h1):
            cover.setdefault((u, h), []).append((r0, r1))
        # a unit in one piece runs both passes; pieces of a cut unit run pass 1 only
        whole = rows is None and (h0, h1) == (0, G)
        assert stages == (P1 | P2 if whole and u > 0 else P1) or (stages == P1 and u == 0)
    # every (unit, head, row) exactly once
    assert sorted(cover) == [(u, h) for u in range(U) for h in range(G)]
    for rr in cover.values():
        rr.sort()
        assert rr[0][0] == 0 and rr[-1][1] == N
        assert all(a[1] == b[0] for a, b in zip(rr, rr[1:]))
    assert any(pc[2] is not None for pc in pieces) == rowed
    if rowed:
        # the last half of every unit's rows (with its k) first, then the
        # second quarter, then the first quarter
        assert len(pieces) == 3 * U
        assert [pc[0] for pc in pieces] == list(range(U)) * 3
        assert all(pc[2][1] == N for pc in pieces[:U]) and all(pc[2][0] == 0 for pc in pieces[2 * U:])
        assert all(pc[3] == P1 for pc in pieces)
    else:
        # unit 0 first, by q-heads; every further unit in one piece
        assert [pc[0] for pc in pieces] == [0] * (len(pieces) - (U - 1)) + list(range(1, U))
