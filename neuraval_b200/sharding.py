"""Sampling over the GPUs of one node, one process per GPU.

TokenSampler.SampleNext (Neuraval/Generation/TokenSampler.cs:10-143) treats
every row on its own, so a batch splits two ways:
  - by rows (`row_range`, `RowShardedSampler`, `PeerRowShardedSampler`): each
    GPU samples its rows with the single-GPU kernels; every GPU then gets all
    rows' tokens and flags, by an NCCL all-gather or through peer memory;
  - by vocabulary (`vocab_range`, `VocabShardedSampler`): each GPU holds its
    columns of every row (a tensor-parallel LM head), reduces them to one
    fixed-size record per row, the records of all GPUs are all-gathered in
    column order (one NCCL collective of rows x 1040 bytes per GPU), and every
    GPU merges them into the same tokens the whole rows give on one GPU.
torch.distributed provides the process group and the collective; NCCL on GPUs,
gloo for the host-side tests.
"""
from __future__ import annotations

import contextlib
from typing import Sequence


def row_range(rows: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous rows of `rank`; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world or rows < 0:
        raise ValueError("bad rows/world/rank")
    base, extra = divmod(rows, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def vocab_range(vocab: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous columns of `rank`: ceil(vocab / world) rounded up to a multiple
    of 4 per shard (16-byte aligned column offsets), the last shard shorter.
    A shard may be empty only when vocab < 4 * world."""
    if world <= 0 or not 0 <= rank < world or vocab <= 0:
        raise ValueError("bad vocab/world/rank")
    step = -(-vocab // world)
    step = (step + 3) // 4 * 4
    lo = min(rank * step, vocab)
    return lo, min(lo + step, vocab)


def gather_records(local, group=None):
    """All-gather a [rows, words] tensor from every rank into [world, rows, words],
    rank order (= column order for vocabulary shards)."""
    import torch
    import torch.distributed as dist
    local = local.contiguous()
    if not dist.is_initialized():
        return local.unsqueeze(0)
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), local, group=group)
    return out


def max_over_ranks(values: Sequence[float], device=None, group=None) -> list[float]:
    """Element-wise maximum of `values` over the ranks (timings: the slowest rank)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return [float(x) for x in t.cpu()]


class RowShardedSampler:
    """Batched SampleNext over a batch split by rows (`row_range`), one range per rank.

    Every rank calls `sample` with its own rows (logits, CSR history and
    uniforms of those rows only) and gets every rank's tokens and flags: one
    all-gather of 2 x ceil(rows / world) int32 per rank (NCCL over NVLink on
    GPUs). The sampling itself needs no exchange: rows are independent
    (TokenSampler.SampleNext samples one row at a time).
    """

    def __init__(self, sampler, rows: int, group=None):
        import torch
        import torch.distributed as dist
        self.sampler = sampler
        self.total_rows = int(rows)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.row_begin, self.row_end = row_range(self.total_rows, self.world, self.rank)
        self.per = -(-self.total_rows // self.world)
        dev = torch.device("cuda", sampler.device)
        # this rank's tokens (row 0) and flags (row 1), padded to `per`
        self.local = torch.zeros((2, self.per), dtype=torch.int32, device=dev)
        self.gathered = torch.zeros((self.world, 2, self.per), dtype=torch.int32, device=dev)

    @property
    def rows(self) -> int:
        return self.row_end - self.row_begin

    def sample(self, logits_rows, hist_ids, hist_offsets, uniforms, params, stream=None) -> None:
        """Asynchronous on `stream` (default: the current stream): samples this
        rank's rows, then all-gathers every rank's tokens and flags."""
        import torch
        import torch.distributed as dist
        if int(logits_rows.shape[0]) != self.rows:
            raise ValueError(f"rank {self.rank} holds rows [{self.row_begin}, {self.row_end}), "
                             f"got {int(logits_rows.shape[0])}")
        ctx = torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext()
        with ctx:
            cur = torch.cuda.current_stream(self.local.device)
            if self.rows > 0:
                self.sampler.sample_rows_device(logits_rows, hist_ids, hist_offsets, uniforms,
                                                params, self.local[0, :self.rows],
                                                self.local[1, :self.rows], None, cur)
            if self.world > 1:
                if dist.get_backend(self.group) == "nccl":
                    dist.all_gather_into_tensor(self.gathered, self.local, group=self.group)
                else:
                    dist.all_gather(list(self.gathered.unbind(0)), self.local, group=self.group)
            else:
                self.gathered[0].copy_(self.local)

    def tokens_flags(self):
        """Every row's (tokens, flags) of the last call, in batch order, as
        device tensors (synchronous only with the stream that sampled)."""
        import torch
        tok, fl = [], []
        for r in range(self.world):
            lo, hi = row_range(self.total_rows, self.world, r)
            tok.append(self.gathered[r, 0, : hi - lo])
            fl.append(self.gathered[r, 1, : hi - lo])
        return torch.cat(tok), torch.cat(fl)


class PeerRowShardedSampler(RowShardedSampler):
    """RowShardedSampler whose gather is done by the library through peer memory
    (each GPU stores its rows' tokens and flags, tagged with the call's epoch,
    into every GPU's gather area over NVLink and waits until its own area holds
    every row of the call) instead of an NCCL all-gather. The process group is used once, to exchange the areas' IPC
    handles."""

    def __init__(self, sampler, rows: int, group=None):
        import torch
        import torch.distributed as dist
        super().__init__(sampler, rows, group)
        mine = sampler.row_gather_setup(self.world, self.rank, self.total_rows)
        n = len(mine)
        local = torch.tensor(list(mine), dtype=torch.uint8)
        if dist.is_initialized() and dist.get_backend(group) == "nccl":
            local = local.cuda(sampler.device)
        everyone = gather_records(local.view(1, n), group)  # [world, 1, n], rank order
        sampler.row_gather_connect(bytes(everyone.view(-1).cpu().tolist()))
        dev = self.local.device
        self.tokens_all = torch.zeros(self.total_rows, dtype=torch.int32, device=dev)
        self.flags_all = torch.zeros(self.total_rows, dtype=torch.int32, device=dev)

    def sample(self, logits_rows, hist_ids, hist_offsets, uniforms, params, stream=None) -> None:
        import torch
        if int(logits_rows.shape[0]) != self.rows:
            raise ValueError(f"rank {self.rank} holds rows [{self.row_begin}, {self.row_end}), "
                             f"got {int(logits_rows.shape[0])}")
        cur = stream if stream is not None else torch.cuda.current_stream(self.local.device)
        self.sampler.sample_rows_gather_device(logits_rows, self.row_begin, hist_ids, hist_offsets,
                                               uniforms, params, self.tokens_all, self.flags_all,
                                               cur)

    def tokens_flags(self):
        return self.tokens_all, self.flags_all


class VocabShardedSampler:
    """Batched SampleNext over a vocabulary split in `vocab_range` shards, one per rank.

    Every rank calls `sample` with its [rows, width] columns; every rank gets
    all rows' tokens. Served: greedy rows and top-k <= 64 (the library returns
    NCB_ERROR_CAPACITY for other options).
    """

    def __init__(self, sampler, vocab: int, group=None):
        import torch.distributed as dist
        self.sampler = sampler
        self.vocab = int(vocab)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.col_begin, self.col_end = vocab_range(self.vocab, self.world, self.rank)
        self.rec_words = sampler.shard_record_bytes // 4
        self._local = None

    @property
    def width(self) -> int:
        return self.col_end - self.col_begin

    def _records(self, rows: int, device):
        import torch
        if self._local is None or self._local.shape[0] < rows or self._local.device != device:
            self._local = torch.empty((rows, self.rec_words), dtype=torch.int32, device=device)
        return self._local[:rows]

    def sample(self, logits_shard, hist_ids, hist_offsets, uniforms, params, tokens,
               flags=None, stream=None) -> None:
        """Asynchronous on `stream` (default: the current stream); the all-gather
        is ordered after the candidate kernel and before the merge."""
        import torch
        rows, width = int(logits_shard.shape[0]), int(logits_shard.shape[1])
        if width != self.width:
            raise ValueError(f"rank {self.rank} holds columns [{self.col_begin}, {self.col_end}),"
                             f" got {width}")
        dev = logits_shard.device
        ctx = torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext()
        with ctx:
            cur = torch.cuda.current_stream(dev)
            local = self._records(rows, dev)
            if width > 0:
                self.sampler.shard_candidates_device(logits_shard, self.vocab, self.col_begin,
                                                     hist_ids, hist_offsets, params, local, cur)
            else:
                local.zero_()  # an empty shard: no candidates, no state
            gathered = gather_records(local, self.group)
            self.sampler.shard_merge_device(gathered, self.world, rows, self.vocab, uniforms,
                                            params, tokens, flags, cur)



class PeerVocabShardedSampler(VocabShardedSampler):
    """VocabShardedSampler whose exchange is done by the library through peer
    memory (records stored into every GPU's exchange area over NVLink as
    epoch-tagged words, waited for by the merge) instead of an NCCL all-gather. The process group is used
    once, to exchange the areas' IPC handles."""

    def __init__(self, sampler, vocab: int, group=None):
        import torch
        import torch.distributed as dist
        super().__init__(sampler, vocab, group)
        mine = sampler.peer_setup(self.world, self.rank)
        n = len(mine)
        local = torch.tensor(list(mine), dtype=torch.uint8)
        if dist.is_initialized() and dist.get_backend(group) == "nccl":
            local = local.cuda(sampler.device)
        everyone = gather_records(local.view(1, n), group)  # [world, 1, n], rank order
        sampler.peer_connect(bytes(everyone.view(-1).cpu().tolist()))

    def sample(self, logits_shard, hist_ids, hist_offsets, uniforms, params, tokens,
               flags=None, stream=None) -> None:
        import torch
        rows, width = int(logits_shard.shape[0]), int(logits_shard.shape[1])
        if width != self.width or width == 0:
            raise ValueError(f"rank {self.rank} holds columns [{self.col_begin}, {self.col_end}),"
                             f" got {width}")
        cur = stream if stream is not None else torch.cuda.current_stream(logits_shard.device)
        self.sampler.shard_push_peer_device(logits_shard, self.vocab, self.col_begin, hist_ids,
                                            hist_offsets, params, cur)
        self.sampler.shard_merge_peer_device(rows, self.vocab, uniforms, params, tokens, flags, cur)
