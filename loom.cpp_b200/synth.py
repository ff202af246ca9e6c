"""Seeded synthetic logits for the logits->token workloads (no dataset is involved).

Every generator draws from a torch.Generator seeded from (seed, stream), on the device it is asked
for, so a workload is reproducible and the oracle and the kernels read identical bytes (the host
copy given to the oracle is the device tensor copied back).

  greedy_decode_step(step)     [1, 151936] f32, N(0, 3^2), plus 8 uniformly placed spikes of +10
  sample_chain(rows)           [rows, 151936] f32, N(0, 3^2); history [rows, 256] uniform in [0, V);
                               u [rows] uniform in [0, 1)
  gemma_vocab(rows)            [rows, 262144] bf16, N(0, 2.5^2) + b[v], b[v] = -1.1 * ln(rank(v)) with
                               rank a seeded permutation of 1..V (the log of a Zipf(1.1) law, shared by
                               all rows); u [rows]
  ctc_frames(n_utt, n_frames)  [n_utt, n_frames, 1025] f32, N(0, 1); per frame +4 on the blank (1024)
                               with probability 0.7, else +4 on a uniform non-blank id
"""
import math

import torch

QWEN3_VOCAB = 151936
GEMMA3_VOCAB = 262144
CTC_CLASSES = 1025
CTC_BLANK = 1024


def _gen(device, seed, stream=0):
    g = torch.Generator(device=device)
    g.manual_seed((int(seed) * 1000003 + int(stream)) & 0x7FFFFFFFFFFFFFFF)
    return g


def greedy_decode_step(step, seed=1, vocab=QWEN3_VOCAB, device="cpu"):
    g = _gen(device, seed, step)
    x = torch.randn(1, vocab, generator=g, device=device, dtype=torch.float32) * 3.0
    pos = torch.randint(0, vocab, (8,), generator=g, device=device)
    x[0, pos] += 10.0
    return x


def sample_chain(rows, seed=2, vocab=QWEN3_VOCAB, hist_len=256, device="cpu"):
    g = _gen(device, seed, rows)
    x = torch.randn(rows, vocab, generator=g, device=device, dtype=torch.float32) * 3.0
    hist = torch.randint(0, vocab, (rows, hist_len), generator=g, device=device, dtype=torch.int64).to(torch.int32)
    u = torch.rand(rows, generator=g, device=device, dtype=torch.float32)
    return x, hist, u


def gemma_vocab(rows, seed=3, vocab=GEMMA3_VOCAB, device="cpu"):
    g = _gen(device, seed, rows)
    rank = torch.randperm(vocab, generator=g, device=device).to(torch.float64) + 1.0
    bias = (-1.1 * torch.log(rank)).to(torch.float32)
    x = torch.randn(rows, vocab, generator=g, device=device, dtype=torch.float32) * 2.5 + bias
    u = torch.rand(rows, generator=g, device=device, dtype=torch.float32)
    return x.to(torch.bfloat16), u


def ctc_frames(n_utt, n_frames, seed=4, n_classes=CTC_CLASSES, blank=CTC_BLANK, device="cpu"):
    g = _gen(device, seed, n_utt * 100003 + n_frames)
    x = torch.randn(n_utt, n_frames, n_classes, generator=g, device=device, dtype=torch.float32)
    is_blank = torch.rand(n_utt, n_frames, generator=g, device=device) < 0.7
    other = torch.randint(0, n_classes - 1, (n_utt, n_frames), generator=g, device=device)
    other = torch.where(other >= blank, other + 1, other)  # a uniform non-blank id
    target = torch.where(is_blank, torch.full_like(other, blank), other)
    x.scatter_add_(2, target.unsqueeze(-1), torch.full((n_utt, n_frames, 1), 4.0, device=device))
    return x


def bf16_bits(t):
    """A bf16 tensor's raw bit patterns as a uint16 numpy array (the oracle's bf16 input form)."""
    return t.contiguous().view(torch.int16).cpu().numpy().view("uint16")


def roofline_bytes(rows, vocab, dtype_bytes=4):
    """Algorithmic bytes of one pass: every logit read once."""
    return rows * vocab * dtype_bytes


assert math.isclose(QWEN3_VOCAB * 4, 607744)
