"""Tensor-parallel partition rules (host mirror of the placement in
csrc/engine.cu: wgd_model_end), and the handle exchange used by the engine.

The reference runs on one device; these rules are this runtime's own:
  * Q/K/V rows split by heads, rank r keeps heads [r*H/tp, (r+1)*H/tp);
  * gate/up rows and the down projection's input columns split in whole GGUF
    blocks of the down matrix (uneven shards allowed, e.g. 84 super-blocks
    over 8 ranks);
  * the attention output projection split by input columns (whole blocks);
  * LM-head rows split in whole 16-row tiles;
  * norms and the embedding replicated.
After the O and down projections the per-rank partial rows are summed
(an allreduce); every rank then holds the same hidden state.
"""
from __future__ import annotations


def part_begin(units: int, r: int, tp: int) -> int:
    """Balanced split: part r is [r*units//tp, (r+1)*units//tp)."""
    return units * r // tp


def ffn_shard(intermediate: int, block: int, r: int, tp: int) -> tuple[int, int]:
    """FFN rows [start, start+count) of rank r, in whole blocks of `block` columns."""
    nblk = intermediate // block
    a, b = part_begin(nblk, r, tp) * block, part_begin(nblk, r + 1, tp) * block
    return a, b - a


def head_shard(heads: int, head_dim: int, r: int, tp: int) -> tuple[int, int]:
    if heads % tp:
        raise ValueError("query and KV head counts must divide by the tensor-parallel size")
    per = heads // tp
    return r * per * head_dim, per * head_dim


def vocab_shard(vocab: int, r: int, tp: int) -> tuple[int, int]:
    tiles = (vocab + 15) // 16
    a = min(vocab, part_begin(tiles, r, tp) * 16)
    b = min(vocab, part_begin(tiles, r + 1, tp) * 16)
    return a, b - a


def torch_exchange(group=None):
    """An all-gather of bytes over torch.distributed, for LoadOptions['exchange']."""
    import torch.distributed as dist

    def exchange(b: bytes):
        out = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, b, group=group)
        return out
    return exchange
