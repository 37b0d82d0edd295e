"""Vocab-parallel sampling across two processes, as the multi-GPU path runs it.

Two ranks (separate processes, gloo process group on 127.0.0.1) each own one
contiguous half of the vocabulary of 64 fp32 rows (the configuration-5 row
distribution).  Each rank builds its shard batch, computes its local top-64
on the GPU (q38s_shard_topk), the ranks all-gather the (value, token) lists
through the process group, and each merges and draws (q38s_shard_merge_sample).
Both ranks must draw the same tokens, and those must equal the canonical
oracle on the unsharded rows (top_k 64, top_p 0.9: the top-64 of the union of
the shards' top-64 is the row's top-64) or be counted boundary cases.

Both processes use the one GPU of the test box; their kernels never wait on
each other (the exchange goes through the host), and the collective is gloo.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROWS, K, WORLD = 64, 64, 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, port, out_dir):
    import sys
    root = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
    sys.path.insert(0, os.path.join(root, "qwen3.8-flash-next-dual-gpu_b200"))
    import torch
    import torch.distributed as dist
    import q38s
    from q38s import synth

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    dev = torch.device("cuda", 0)
    V = synth.VOCAB
    w = V // WORLD
    col0 = rank * w
    spec = synth.cfg5_spec(rows=ROWS)
    configs = [q38s.config_v2(top_k=64, top_p=0.9, temperature=0.8, repetition_penalty=1.1,
                              seed=int(spec.seed[r])) for r in range(ROWS)]
    sb = q38s.Batch(V, configs, shard=(col0, w))
    sb.commit_tokens([h[(h >= col0) & (h < col0 + w)] for h in spec.histories])
    host = np.stack([synth.cfg5_row(r)[col0:col0 + w] for r in range(ROWS)])
    local = sb.shard_topk(torch.from_numpy(host).to(dev), K)
    torch.cuda.synchronize()
    parts = [torch.zeros_like(local.cpu()) for _ in range(WORLD)]
    dist.all_gather(parts, local.cpu())  # shards in rank (column) order
    gathered = torch.cat(parts).to(dev)
    dec = sb.decode_decisions(sb.shard_merge_sample(gathered, WORLD, K))
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"rank{rank}.npy"),
            np.stack([dec["token"], dec["status"]]).astype(np.int64))
    dist.barrier()
    dist.destroy_process_group()


def test_two_ranks_gather_merge_match_the_unsharded_oracle(cuda, tmp_path):
    import torch.multiprocessing as mp
    import oracle as O
    from helpers import is_boundary
    from q38s import synth

    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, port, str(tmp_path))) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f"rank process exit code {p.exitcode}"
    r0 = np.load(tmp_path / "rank0.npy")
    r1 = np.load(tmp_path / "rank1.npy")
    assert (r0 == r1).all(), "ranks drew different tokens"
    assert (r0[1] == 0).all()
    spec = synth.cfg5_spec(rows=ROWS)
    boundary = 0
    for r in range(ROWS):
        row = synth.cfg5_row(r)
        counts = np.bincount(spec.histories[r], minlength=synth.VOCAB).astype(np.uint32)
        p = O.make_params(top_k=64, top_p=0.9, temperature=0.8, repetition_penalty=1.1,
                          rng_state=int(spec.seed[r]))
        o = O.prepare_row(p, row, counts, (), O.TIE_CANONICAL, cap=64)
        if o.token != r0[0][r]:
            assert is_boundary(o, 0.9), f"row {r}: {r0[0][r]} vs oracle {o.token}"
            boundary += 1
    print(f"vocab-parallel over 2 ranks: {ROWS} rows, boundary cases {boundary}")
    assert boundary <= 1
