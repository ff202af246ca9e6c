"""Multi-GPU plumbing of the logits->token stage: one process per GPU, torch.distributed for the
exchange (NCCL over NVLink on B200; gloo works for the same calls on CPU tensors).

Two ways to spread the work:
  - rows: rank g samples rows [g*B/G, (g+1)*B/G) of the batch. Rows are independent, so there is no
    exchange at all; each rank keeps its own results (or gathers them, if a caller wants them in one
    place).
  - vocabulary: rank g owns ids [g*V/G, (g+1)*V/G) of every row, runs loom_sample_shard_partial on
    its slice, all-gathers the per-row records (loom_shard_record_bytes(k) bytes each: the shard's
    top-k (value, global id) and its partial max / sum-exp), and merges them with
    loom_sample_shard_merge. Every rank ends with the full result.
"""
import torch
import torch.distributed as dist


def split(n, world, rank):
    """[lo, hi) of the rank-th of `world` near-equal contiguous pieces of range(n)."""
    return n * rank // world, n * (rank + 1) // world


def gather_records(local, group=None):
    """All-gather equal-size uint8 record buffers: returns [world, local.numel()] in rank order."""
    world = dist.get_world_size(group)
    out = torch.empty(world, local.numel(), dtype=local.dtype, device=local.device)
    if local.is_cuda:
        dist.all_gather_into_tensor(out.view(-1), local.contiguous().view(-1), group=group)
    else:
        parts = list(out.unbind(0))
        dist.all_gather(parts, local.contiguous().view(-1), group=group)
    return out


def sample_vocab_sharded(x_shard, vocab_offset, vocab_total, u, temperature, repetition_penalty=1.0, top_k=64,
                         top_p=1.0, history=None, want_logp=False, group=None, workspace=None, stream=None):
    """The sampling chain over a vocabulary split across the ranks of `group`.

    x_shard: this rank's [rows, shard_vocab] CUDA slice; u: [rows] uniforms, identical on every rank.
    Returns (ids, probs[, logp]) for all rows, identical on every rank.
    """
    import loom_select as sel

    rows = x_shard.shape[0]
    rb = sel.shard_record_bytes(top_k)
    local = torch.empty(rows * rb, dtype=torch.uint8, device=x_shard.device)
    sel.shard_partial_into(x_shard, local, vocab_offset, vocab_total, temperature, repetition_penalty, top_k, top_p,
                           history=history, workspace=workspace, stream=stream)
    records = gather_records(local, group)
    world = records.shape[0]
    ids = torch.empty(rows, dtype=torch.int32, device=x_shard.device)
    prob = torch.empty(rows, dtype=torch.float32, device=x_shard.device)
    logp = torch.empty(rows, dtype=torch.float32, device=x_shard.device) if want_logp else None
    sel.shard_merge_into(records, world, rows, u, ids, prob, temperature, top_k, top_p, out_logp=logp, stream=stream)
    return (ids, prob, logp) if want_logp else (ids, prob)
