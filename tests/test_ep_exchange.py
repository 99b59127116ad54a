"""Expert-parallel exchange on CPU: two and four gloo ranks, oracle dispatch plans, a stand-in expert.

The device kernels of the dispatch plan / pack / combine are checked on the GPU against the same
oracle (tests/test_gpu_ep.py). Here the host logic runs for real: the count all-to-all, the ragged
row and slot all-to-alls and the return trip, with every rank's tokens routed to experts spread over
all ranks. The stand-in expert multiplies a row by (global id + 1), so a misrouted row, slot or
return lands on a visibly wrong value.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_inputs(rank, T, H, k, E):
    rng = np.random.default_rng(100 + rank)
    x = rng.normal(0, 1, (T, H)).astype(np.float32)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.uint32)
    ids[rng.random((T, k)) < 0.1] = 0xFFFFFFFF  # some empty slots
    w = rng.random((T, k)).astype(np.float32)
    return x, ids, w


def _worker(rank, world, port, T, H, k, epr, out_dir):
    import torch.distributed as dist

    from moe_b200 import ep
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        E = epr * world
        x, ids, w = _rank_inputs(rank, T, H, k, E)
        rank_counts, token_rows, send_token, send_ids, send_w = O.ep_dispatch_plan(ids, w, epr, world)
        send_x = torch.from_numpy(x[send_token])
        sc, rc = ep.exchange_counts(torch.from_numpy(rank_counts), None)
        recv_x = ep.exchange_rows(send_x, sc, rc)
        meta = torch.from_numpy(np.concatenate([send_ids.view(np.int32), send_w.view(np.int32)], axis=1))
        recv_meta = ep.exchange_rows(meta, sc, rc)
        rid = recv_meta[:, :k].numpy().view(np.uint32)
        rw = recv_meta[:, k:].contiguous().numpy().view(np.float32)
        # stand-in local expert: row * (global id + 1), weighted, slots in order
        gid = np.where(rid == 0xFFFFFFFF, 0, rid.astype(np.int64) + rank * epr)
        scale = np.where(rid == 0xFFFFFFFF, 0.0, rw * (gid + 1)).sum(1)
        y_recv = torch.from_numpy((recv_x.numpy() * scale[:, None]).astype(np.float32))
        y_back = ep.exchange_rows(y_recv, rc, sc)
        y = O.ep_combine(y_back.numpy(), token_rows)
        valid = ids != 0xFFFFFFFF
        want = x * np.where(valid, w * (ids.astype(np.int64) + 1), 0.0).sum(1)[:, None]
        np.save(os.path.join(out_dir, f"r{rank}.npy"), np.stack([y, want]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ep_exchange_routes_rows_and_results(world, tmp_path):
    import torch.multiprocessing as mp

    T, H, k, epr = 37, 24, 4, 3
    mp.spawn(_worker, args=(world, _free_port(), T, H, k, epr, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        y, want = np.load(tmp_path / f"r{r}.npy")
        np.testing.assert_allclose(y, want, rtol=1e-5, atol=1e-5)


def test_oracle_dispatch_plan_properties():
    from oracle import oracle as O

    rng = np.random.default_rng(0)
    T, k, epr, world = 50, 8, 4, 8
    ids = np.stack([rng.permutation(epr * world)[:k] for _ in range(T)]).astype(np.uint32)
    w = rng.random((T, k)).astype(np.float32)
    rank_counts, token_rows, send_token, send_ids, send_w = O.ep_dispatch_plan(ids, w, epr, world)
    # every (token, slot) lands exactly once, on its owner, with its weight and local id
    seen = np.zeros((T, k), dtype=int)
    for row in range(send_token.size):
        t = send_token[row]
        r = int(np.searchsorted(np.cumsum(rank_counts), row, side="right"))
        assert token_rows[t, r] == row
        for j in range(k):
            if send_ids[row, j] != O.ID_NONE:
                assert ids[t, j] // epr == r and send_ids[row, j] == ids[t, j] - r * epr
                assert send_w[row, j] == w[t, j]
                seen[t, j] += 1
    assert (seen == 1).all()
    # rows of a rank are in token order
    starts = np.concatenate([[0], np.cumsum(rank_counts)])
    for r in range(world):
        assert np.all(np.diff(send_token[starts[r]:starts[r + 1]]) > 0)
