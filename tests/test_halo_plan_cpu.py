"""The torus halo plan (``mtorus.parallel.symm.halo_plan``) that drives the
peer-store neighbour exchange, simulated on the CPU: every rank "stores" its id into
slot nbr_slot[k] of rank nbr_rank[k]; afterwards slot j of every rank must hold the
id of its neighbour in direction j (+x, -x, +y, -y, ...), with no slot written twice
-- including 2-wide axes, where the +x and -x neighbour is the same rank."""
import pytest
import torch

from mtorus.core.topology import MeshTorusHybrid
from mtorus.parallel.symm import halo_plan


@pytest.mark.parametrize("dims", [(2, 4), (4, 4), (2, 2), (3, 5), (2, 2, 2), (4, 2, 3)])
def test_every_slot_receives_its_direction(dims):
    topo = MeshTorusHybrid.new_2d(*dims, 1) if len(dims) == 2 else MeshTorusHybrid.new_3d(*dims, 1)
    n = 1
    for d in dims:
        n *= d
    nslots = 2 * len(dims)
    recv = torch.full((n, nslots), -1, dtype=torch.int64)
    for r in range(n):
        nr, ns = halo_plan(topo, r, "cpu")
        assert nr.numel() == ns.numel() == nslots
        for q, j in zip(nr.tolist(), ns.tolist()):
            assert recv[q, j] == -1, f"slot {j} of rank {q} written twice"
            recv[q, j] = r
    for q in range(n):
        nbrs = topo.rank_to_coords(q).neighbors(topo.dims)
        for j, (c, _axis) in enumerate(nbrs):
            assert recv[q, j] == topo.node_rank(c), (q, j)
