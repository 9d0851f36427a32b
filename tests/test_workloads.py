"""Per-unit input draws are exact slices of the workload protocol.

``make_unit_inputs`` redraws each (batch, kv-head) unit from the CPU generator
state at its place in ``make_inputs``' stream, so that a multi-GPU rank draws
only its own units yet sees the very values the single-GPU run and the golden
fixtures use.  The Llama-3-70B N=131072 states are stored
(``workload_states.json``); the links of that chain are checked here.
"""

import torch
import pytest

from kvblockmass_b200 import workloads as wl
from kvblockmass_b200.workloads import WORKLOADS, make_inputs, make_unit_inputs


@pytest.mark.parametrize("name", sorted(WORKLOADS))
def test_unit_inputs_are_slices_of_the_full_draw(name):
    w = WORKLOADS[name]
    n = 384
    q, k, _, _ = make_inputs(w, N=n)
    G = w.G
    last = w.units - 1
    for ub, ue in [(0, w.Hkv), (1, min(3, w.Hkv)), (last, last + 1), (w.Hkv * (w.B - 1), w.Hkv * w.B)]:
        b, g0 = divmod(ub, w.Hkv)
        g1 = g0 + (ue - ub)
        qu, ku = make_unit_inputs(w, ub, ue, N=n, threads=2)
        assert qu.dtype == w.dtype and qu.shape == (1, (ue - ub) * G, n, w.D)
        assert torch.equal(qu, q[b:b + 1, g0 * G:g1 * G]), (ub, ue)
        assert torch.equal(ku, k[b:b + 1, g0:g1]), (ub, ue)


def test_unit_ranges_must_stay_in_one_batch_entry():
    w = WORKLOADS["batched_masked_n16k"]
    with pytest.raises(ValueError):
        make_unit_inputs(w, w.Hkv - 1, w.Hkv + 1, N=128)
    with pytest.raises(ValueError):
        make_unit_inputs(w, 0, w.units + 1, N=128)


def test_stored_70b_states_are_the_stream():
    """The stored states start at the seed and each link is one unit's draw:
    spot-check the first and last links of the q chain and the k chain."""
    w = WORKLOADS["llama3_70b_n128k"]
    st = wl._stored_states(w, w.N)
    if st is None:
        pytest.skip("no stored states for this torch version (they would be recomputed)")
    assert len(st["q"]) == w.units and len(st["k"]) == w.units
    assert torch.equal(st["q"][0], torch.Generator().manual_seed(w.seed).get_state())
    for chain, nxt, shape in [(st["q"][0], st["q"][1], (1, w.G, w.N, w.D)),
                              (st["q"][-1], st["k"][0], (1, w.G, w.N, w.D)),
                              (st["k"][-1], st["extra"], (1, 1, w.N, w.D))]:
        g = torch.Generator()
        g.set_state(chain)
        torch.randn(*shape, generator=g, dtype=torch.float32)
        assert torch.equal(g.get_state(), nxt)
