"""The C5 GPT workload's host logic on CPU: Zipf token ids, the parameter count of the benchmark
configuration, and data-parallel training over two ``gloo`` ranks, which must end with the same
parameters on both ranks as one process training on the two ranks' batches together.

Attention here is a plain fp32 PyTorch restatement of Born attention (the native op is CUDA only).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from quantumdlblocks_b200.gpt import BornGPT, GPTConfig, param_count, train_step, zipf_tokens

TINY = GPTConfig(vocab_size=97, d_model=64, n_layers=2, n_heads=4, seq_len=16)


def born_eager(q, k, v, scale, is_causal=True, eps=1e-12):
    """fp32 Born attention: relu(scale q.k)^2 masked causally, rows normalised by sum + eps
    (computed in fp32 also under autocast; returned in v's dtype)."""
    with torch.autocast(q.device.type, enabled=False):
        sc = scale.float() if isinstance(scale, torch.Tensor) else scale
        a = torch.relu(torch.matmul(q.float(), k.float().transpose(-1, -2)) * sc)
        T = q.shape[-2]
        if is_causal:
            a = a * torch.ones(T, T, dtype=torch.bool, device=q.device).tril()
        p = a * a
        return (torch.matmul(p, v.float()) / (p.sum(-1, keepdim=True) + eps)).to(v.dtype)


def test_zipf_tokens_range_and_skew():
    t = zipf_tokens(4, 255, 1000, seed=3)
    assert t.shape == (4, 256) and t.dtype == np.int64
    assert t.min() >= 0 and t.max() < 1000
    counts = np.bincount(t.ravel(), minlength=1000)
    assert counts[0] > counts[1] > counts[10]  # rank 1 is the most frequent id
    assert np.array_equal(t, zipf_tokens(4, 255, 1000, seed=3))


def test_benchmark_config_has_127m_parameters():
    with torch.device("meta"):
        model = BornGPT(GPTConfig(), attention=born_eager)
    n = param_count(model)
    assert 126e6 < n < 128e6, n  # 51.5 M tied embedding + 6 x 12.6 M blocks


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch(rank: int) -> torch.Tensor:
    return torch.from_numpy(zipf_tokens(3, TINY.seq_len, TINY.vocab_size, seed=50 + rank))


def _flat(model) -> torch.Tensor:
    return torch.cat([p.detach().reshape(-1) for p in model.parameters()])


def _rank_main(rank, world, port, out_path):
    import torch.distributed as dist

    from quantumdlblocks_b200.gpt import make_ddp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        model = BornGPT(TINY, attention=born_eager)
        net = make_ddp(model, torch.device("cpu"))
        opt = torch.optim.SGD(model.parameters(), lr=0.5)  # linear in the averaged gradient
        for _ in range(2):
            train_step(net, opt, _batch(rank), autocast_dtype=None)
        mine = _flat(model)
        other = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(other, mine)
        if rank == 0:
            torch.save({"ranks": other}, out_path)
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_two_gloo_ranks_train_like_one_process_on_both_batches(tmp_path):
    import torch.multiprocessing as mp

    out_path = str(tmp_path / "params.pt")
    mp.spawn(_rank_main, args=(2, _free_port(), out_path), nprocs=2, join=True)
    ranks = torch.load(out_path)["ranks"]
    assert torch.equal(ranks[0], ranks[1])  # the all-reduce kept the replicas identical
    torch.manual_seed(0)
    model = BornGPT(TINY, attention=born_eager)
    init = _flat(model).clone()
    opt = torch.optim.SGD(model.parameters(), lr=0.5)
    both = torch.cat([_batch(0), _batch(1)])
    for _ in range(2):
        train_step(model, opt, both, autocast_dtype=None)
    moved = (ranks[0] - init).abs().max().item()
    assert moved > 1e-3  # the steps changed the parameters
    # fp32 sums over one batch of 6 and two averaged batches of 3 differ in their last bits; a
    # wrong reduction (a sum instead of the mean, one rank's gradient) would miss by ~lr * grad
    torch.testing.assert_close(ranks[0], _flat(model), rtol=0, atol=2e-5)


def test_padded_head_matches_unpadded_model():
    """Padding the tied head to a multiple of 64 rows (masked at -inf) changes no loss or gradient."""
    import dataclasses

    torch.manual_seed(1)
    padded = BornGPT(TINY, attention=born_eager)
    plain = BornGPT(dataclasses.replace(TINY, pad_vocab_to=1), attention=born_eager)
    assert padded.emb.num_embeddings == 128 and plain.emb.num_embeddings == TINY.vocab_size
    sd = padded.state_dict()
    sd["emb.weight"] = sd["emb.weight"][:TINY.vocab_size]
    plain.load_state_dict(sd)
    tok = _batch(0)
    lp = padded(tok[:, :-1], tok[:, 1:])
    lu = plain(tok[:, :-1], tok[:, 1:])
    lp.backward()
    lu.backward()
    torch.testing.assert_close(lp, lu, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(padded.emb.weight.grad[:TINY.vocab_size], plain.emb.weight.grad, rtol=1e-5, atol=1e-7)
    assert padded.emb.weight.grad[TINY.vocab_size:].abs().max() == 0
    assert param_count(padded) == param_count(plain)
