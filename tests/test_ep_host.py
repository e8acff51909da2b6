"""Expert-parallel host orchestration on gloo CPU ranks (world size 2).

The extension's calls are replaced by the oracle's CPU stand-ins
(oracle/ep_oracle.py), so what runs here is the layer's own logic: routing
to ranks, split sizes, the three all-to-alls and the combine.  Checked against
the single-device oracle on the same global weights; an injected rank failure
(a rank raising before the exchange) must end the other rank's collective
with an error, not a hang.
"""
import socket

import pytest
import torch.multiprocessing as mp

from tests import _ep_worker


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(scenario, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_ep_worker.cpu_rank, args=(r, world, port, q, scenario))
             for r in range(world)]
    for p in procs:
        p.start()
    out = []
    try:
        for _ in range(world):
            out.append(q.get(timeout=timeout))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join()
    return sorted(out, key=lambda r: r[1])


@pytest.mark.parametrize("scenario", ["all", "mask"])
def test_ep_two_ranks_match_single_device_oracle(scenario):
    res = _run(scenario)
    for status, rank, val, sc, rc in res:
        assert status == "ok", (rank, val)
        assert val < 1e-5, (rank, val)
    # what rank 0 sends to rank 1 is what rank 1 receives from rank 0
    assert res[0][3][1] == res[1][4][0]
    assert res[1][3][0] == res[0][4][1]


def test_ep_four_ranks_deduplicated_rows_match_single_device_oracle():
    """World 4: one send row per (token, destination rank) with up to P = 2 of the
    token's selections on that rank; every rank's output equals the oracle and
    what rank i sends to rank j is what j receives from i."""
    res = _run("all", world=4)
    for status, rank, val, sc, rc in res:
        assert status == "ok", (rank, val)
        assert val < 1e-5, (rank, val)
    for i in range(4):
        for j in range(4):
            assert res[i][3][j] == res[j][4][i]


@pytest.mark.parametrize("world", [2, 4])
def test_fixed_segments_need_no_counts_and_match_the_oracle(world):
    """Fixed all-to-all segments (equal splits, padding rows travel): no count
    exchange, every rank's output equals the single-device oracle."""
    res = _run("fixed", world=world)
    for status, rank, val, sc, rc in res:
        assert status == "ok", (rank, val)
        assert val < 1e-5, (rank, val)
        assert len(sc) == world and all(0 <= c <= 16 for c in sc)


def test_injected_rank_failure_ends_the_collective_with_an_error():
    res = _run("fail", timeout=90)
    by_rank = {r[1]: r for r in res}
    assert by_rank[1][0] == "error" and "injected" in by_rank[1][2]
    assert by_rank[0][0] == "error"


@pytest.mark.parametrize("chunks", [1, 3])
def test_single_rank_dispatch_path_without_a_process_group(chunks):
    """One rank, no process group, the dispatch path forced: the exchanges
    degenerate to copies and the result equals the single-device oracle."""
    import torch
    from oracle import moe_oracle as O
    from oracle.ep_oracle import CpuEpBackend
    from project_chronos_b200.ep import ExpertParallelMoE
    E, k, H, F, S = 8, 2, 32, 16, 1
    w = _ep_worker._weights(E, H, F, S)
    x = torch.randn(11, H, generator=torch.Generator().manual_seed(3))
    m = ExpertParallelMoE.from_stacked(_ep_worker._cfg(E, k, H, F, S), w["router"], w["gate"], w["up"],
                                       w["down"], w["sh_gate"], w["sh_up"], w["sh_down"],
                                       backend=CpuEpBackend(), dispatch_single_rank=True)
    m.chunks = chunks
    mask = torch.tensor([1, 1, 0, 1, 1, 1, 0, 1], dtype=torch.float32)
    y = m(x, available_expert_mask=mask)
    ref, _, _, _ = O.moe_forward(x.numpy(), w["router"].numpy(), w["gate"].numpy(), w["up"].numpy(),
                                 w["down"].numpy(), w["sh_gate"].numpy(), w["sh_up"].numpy(),
                                 w["sh_down"].numpy(), k, True, avail=mask.numpy())
    assert O.rel_l2(y.numpy(), ref) < 1e-5
    assert m.last_send_counts == m.last_recv_counts
