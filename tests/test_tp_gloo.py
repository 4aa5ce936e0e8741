"""The tensor-parallel split on CPU with world_size-2 gloo ranks: each rank
computes its shard of the column-split (Q/K/V, gate/up) and row-split (O,
down) projections with the CPU oracle, an allreduce sums the row-split
partials, and the result must equal the unsharded product — for an even split
and for the uneven block split of a Gemma-3-27B-like FFN (84 blocks over 8
ranks, here 21 blocks over 2... and 5 blocks over 2)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from webgpu_b200 import synth, tp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, ttype, rows, cols, nblk_ffn, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        be, bb = synth.BLOCK[ttype]
        x = synth.normal(cols, 31, 1)
        # column split (rows of W): gate/up-like matrix with `rows` rows in whole blocks
        w_up = synth.random_blocks(ttype, rows * cols // be, seed=31, stream=2).reshape(rows, -1)
        a, n = tp.ffn_shard(rows, be, rank, world)
        y_shard = oracle.matmul(w_up[a:a + n].reshape(-1), ttype, n, cols, x, 1)[0]
        parts = [None] * world
        dist.all_gather_object(parts, (a, y_shard))
        y_cat = np.zeros(rows)
        for s0, ys in parts:
            y_cat[s0:s0 + len(ys)] = ys
        full_up = oracle.matmul(w_up.reshape(-1), ttype, rows, cols, x, 1)[0]
        # row split (columns of W): down-like matrix [cols x rows], input = y (the FFN activation)
        act = full_up.astype(np.float32)
        w_dn = synth.random_blocks(ttype, cols * rows // be, seed=31, stream=3).reshape(cols, -1)
        rb = rows // be * bb
        c0, cn = a // be * bb, n // be * bb
        dn_cols = w_dn[:, c0:c0 + cn].reshape(-1)
        partial = oracle.matmul(np.ascontiguousarray(dn_cols), ttype, cols, n, act[a:a + n], 1)[0]
        t = torch.from_numpy(partial.copy())
        dist.all_reduce(t)
        full_dn = oracle.matmul(w_dn.reshape(-1), ttype, cols, rows, act, 1)[0]
        q.put((rank, float(np.max(np.abs(y_cat - full_up))), float(np.max(np.abs(t.numpy() - full_dn)) / np.max(np.abs(full_dn)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ttype,rows,cols", [(12, 5 * 256, 512), (12, 4 * 256, 256), (8, 7 * 32, 128)])
def test_tp_split_equals_unsharded(ttype, rows, cols):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, ttype, rows, cols, 0, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, col_err, row_err in results:
        assert col_err == 0.0, (rank, col_err)  # column split reproduces the rows exactly
        assert row_err < 1e-12, (rank, row_err)  # row split + allreduce: f64 reassociation only


def test_partition_rules():
    # Gemma-3-27B FFN: 21504 = 84 super-blocks over 8 ranks -> 10/11 blocks, covering all rows
    spans = [tp.ffn_shard(21504, 256, r, 8) for r in range(8)]
    assert sum(n for _, n in spans) == 21504
    assert all(n in (2560, 2816) for _, n in spans)
    assert [a for a, _ in spans] == sorted(a for a, _ in spans)
    # Llama-3-8B: 14336 / 8 = 7 super-blocks each
    assert {tp.ffn_shard(14336, 256, r, 8)[1] for r in range(8)} == {1792}
    # vocab split in whole tiles of 16 rows
    v = [tp.vocab_shard(128256, r, 8) for r in range(8)]
    assert sum(n for _, n in v) == 128256 and all(a % 16 == 0 for a, _ in v)
    assert tp.head_shard(32, 128, 3, 8) == (3 * 4 * 128, 4 * 128)
    with pytest.raises(ValueError):
        tp.head_shard(14, 64, 0, 4)
