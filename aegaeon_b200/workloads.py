"""Seeded synthetic workloads with the shapes of the benchmark configurations.

Each builder returns plain Python data (shapes, id lists); the benchmark and
tests allocate the tensors.  Block ids come from ``torch.randperm`` on a seeded
CPU generator; cache contents from a seeded device generator.

  cfg1  Qwen3-4B:        36 layers, K and V [1024, 16, 8, 128] bf16, N(0,1);
                         256 blocks out to slots 0..255, then back in to a
                         fresh permutation.
  cfg2  Llama-2-7B:      32 layers, K/V [4096, 16, 32, 128] fp16, U(-2,2);
                         1024 blocks out and 1024 in per step.
  cfg3  Qwen2.5-7B P->D: 28 layers, 4 kv heads, 128 dim, bf16; 8 requests per
                         GPU pair, prompt lengths U{512..8192}.
  cfg4  switch overlap:  2048-block cfg2 swap-in + Qwen1.5-14B-shaped bf16
                         weights (TP-2 shard) in 64 MiB chunks.
  cfg5  Qwen1.5-MoE:     24 layers, 16 kv heads, 128 dim, bf16; 16384-entry
                         mapping, half in contiguous runs of length 1..32.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List

import torch


@dataclass
class KVShape:
    name: str
    layers: int
    kv_heads: int
    head_dim: int
    dtype: torch.dtype
    block_size: int = 16
    num_blocks: int = 1024
    dist: str = "normal"  # "normal" N(0,1) | "uniform2" U(-2,2)

    @property
    def page_bytes(self) -> int:
        """Bytes of one block of one K or V tensor (P * H * D * e)."""
        return self.block_size * self.kv_heads * self.head_dim * torch.tensor(
            [], dtype=self.dtype).element_size()

    @property
    def num_segments(self) -> int:
        return 2 * self.layers  # separate K and V tensors per layer

    @property
    def composite_bytes(self) -> int:
        return self.num_segments * self.page_bytes


CFG1 = KVShape("Qwen3-4B", 36, 8, 128, torch.bfloat16, num_blocks=1024, dist="normal")
CFG2 = KVShape("Llama-2-7B", 32, 32, 128, torch.float16, num_blocks=4096, dist="uniform2")
CFG3 = KVShape("Qwen2.5-7B", 28, 4, 128, torch.bfloat16, num_blocks=4096, dist="normal")
CFG5 = KVShape("Qwen1.5-MoE-A2.7B", 24, 16, 128, torch.bfloat16, num_blocks=16384,
               dist="normal")


def fill_segment(t: torch.Tensor, shape: KVShape, gen: torch.Generator) -> None:
    """Fill a uint8 page tensor with values of the configured distribution."""
    v = t.view(shape.dtype)
    if shape.dist == "uniform2":
        v.uniform_(-2.0, 2.0, generator=gen)
    else:
        v.normal_(0.0, 1.0, generator=gen)


def randperm(n: int, seed: int) -> List[int]:
    return torch.randperm(n, generator=torch.Generator().manual_seed(seed)).tolist()


def swap_step_ids(num_blocks: int, per_direction: int, step: int, seed: int = 0):
    """Disjoint (out_ids, in_ids) device block ids for one cfg2 step."""
    p = randperm(num_blocks, seed * 1_000_003 + step)
    return p[:per_direction], p[per_direction:2 * per_direction]


@dataclass
class MigrationPlan:
    prompt_lengths: List[int]
    blocks_per_request: List[int]
    source_ids: List[int]
    target_ids: List[int]

    @property
    def num_blocks(self) -> int:
        return len(self.source_ids)


def migration_plan(shape: KVShape, requests: int = 8, seed: int = 0, pair: int = 0,
                   lo: int = 512, hi: int = 8192) -> MigrationPlan:
    """cfg3: prompt lengths U{lo..hi}, ceil(len/16) blocks each, random
    source / destination tables drawn from each GPU's pool."""
    g = torch.Generator().manual_seed(seed * 7919 + pair)
    lengths = torch.randint(lo, hi + 1, (requests,), generator=g).tolist()
    blocks = [math.ceil(n / shape.block_size) for n in lengths]
    total = sum(blocks)
    if total > shape.num_blocks:
        raise ValueError(f"pool of {shape.num_blocks} blocks too small for {total}")
    src = torch.randperm(shape.num_blocks, generator=g)[:total].tolist()
    dst = torch.randperm(shape.num_blocks, generator=g)[:total].tolist()
    return MigrationPlan(lengths, blocks, src, dst)


def fragmented_mapping(num_entries: int, num_blocks: int, seed: int = 0):
    """cfg5: device ids of `num_entries` entries, half in contiguous runs of
    length U{1..32}, half isolated random blocks; host slots 0..n-1."""
    g = torch.Generator().manual_seed(seed)
    used = set()
    ids: List[int] = []
    half = num_entries // 2
    while len(ids) < half:
        run = int(torch.randint(1, 33, (1,), generator=g))
        run = min(run, half - len(ids))
        for _ in range(64):
            start = int(torch.randint(0, num_blocks - run, (1,), generator=g))
            if all((start + k) not in used for k in range(run)):
                break
        else:
            continue
        for k in range(run):
            used.add(start + k)
            ids.append(start + k)
    free = [b for b in torch.randperm(num_blocks, generator=g).tolist() if b not in used]
    singles = free[: num_entries - len(ids)]
    # interleave: runs and singles in a random order of "pieces"
    pieces: List[List[int]] = []
    i = 0
    while i < len(ids):
        j = i + 1
        while j < len(ids) and ids[j] == ids[j - 1] + 1:
            j += 1
        pieces.append(ids[i:j])
        i = j
    pieces += [[b] for b in singles]
    order = torch.randperm(len(pieces), generator=g).tolist()
    out = [b for k in order for b in pieces[k]]
    return out, list(range(num_entries))


@dataclass
class WeightShard:
    """Qwen1.5-14B-shaped bf16 weights, every 2-D matrix halved (one TP-2
    shard): 40 layers, hidden 5120, intermediate 13696, vocab 152064."""

    layers: int = 40
    hidden: int = 5120
    intermediate: int = 13696
    vocab: int = 152064
    tp: int = 2
    tensors: List[int] = field(default_factory=list)

    def __post_init__(self):
        h, i, v, tp = self.hidden, self.intermediate, self.vocab, self.tp
        per_layer = [
            3 * h * h // tp + 3 * h // tp,  # qkv proj (+bias)
            h * h // tp,                     # o proj
            2 * h * i // tp,                 # gate + up
            i * h // tp,                     # down
            2 * h,                           # two norms (replicated)
        ]
        self.tensors = [v * h // tp] + per_layer * self.layers + [h, v * h // tp]

    @property
    def nbytes(self) -> int:
        return 2 * sum(self.tensors)
