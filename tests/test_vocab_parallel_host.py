"""Host side of vocab-parallel sampling, two gloo ranks on the CPU.

The multi-GPU path gathers every rank's local top-k list (value, token) in
rank order, so that shard s's list for row r sits at [(s * rows + r) * k],
and every rank merges the union into the row's global top-k.  This checks
that contract without a GPU: each rank computes its shard's lists with the
CPU oracle (oracle.shard_topk: penalties on the shard's own columns, global
token ids), the ranks all-gather through a gloo process group, and the merge
of the gathered lists in canonical order (value desc, token asc) must equal
the top-k of the unsharded row.
"""
import os
import socket

import numpy as np

ROWS, K, WORLD, V = 6, 64, 2, 20_000


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rows():
    rng = np.random.default_rng(55)
    x = rng.normal(0, 2.5, (ROWS, V)).astype(np.float32)
    hists = [rng.integers(0, V, 300).astype(np.int32) for _ in range(ROWS)]
    return x, hists


def _params(O):
    return O.make_params(top_k=K, top_p=0.9, temperature=0.8, repetition_penalty=1.1,
                         rng_state=1)


def _rank_main(rank, port, out_dir):
    import sys
    root = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
    sys.path.insert(0, os.path.join(root, "oracle"))
    import torch
    import torch.distributed as dist
    import oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    x, hists = _rows()
    w = V // WORLD
    col0 = rank * w
    vals = np.zeros((ROWS, K), np.float32)
    toks = np.zeros((ROWS, K), np.int32)
    for r in range(ROWS):
        counts = np.bincount(hists[r], minlength=V)[col0:col0 + w].astype(np.uint32)
        v, t = O.shard_topk(V, col0, _params(O), x[r, col0:col0 + w], K, counts)
        vals[r, :len(v)], toks[r, :len(t)] = v, t
    local = torch.from_numpy(np.stack([vals.view(np.int32), toks], axis=-1).reshape(-1))
    parts = [torch.zeros_like(local) for _ in range(WORLD)]
    dist.all_gather(parts, local)
    np.save(os.path.join(out_dir, f"gathered{rank}.npy"), torch.cat(parts).numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gather_layout_and_merge(tmp_path):
    import torch.multiprocessing as mp
    import oracle as O

    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, port, str(tmp_path))) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    g0 = np.load(tmp_path / "gathered0.npy")
    g1 = np.load(tmp_path / "gathered1.npy")
    assert (g0 == g1).all(), "ranks gathered different lists"
    lists = g0.reshape(WORLD, ROWS, K, 2)
    x, hists = _rows()
    for r in range(ROWS):
        cand = [(float(np.int32(v).view(np.float32)), int(t))
                for s in range(WORLD) for v, t in lists[s, r] if t >= 0]
        merged = sorted(cand, key=lambda vt: (-vt[0], vt[1]))[:K]
        counts = np.bincount(hists[r], minlength=V).astype(np.uint32)
        o = O.prepare_row(_params(O), x[r], counts, (), O.TIE_CANONICAL, cap=K)
        assert [t for _, t in merged] == list(o.cand_tokens[:K]), f"row {r}"
        assert np.allclose([v for v, _ in merged], o.cand_values[:K], rtol=0, atol=0)
