"""GPU parity of the vocabulary-shard greedy verify kernels (nva_shard_argmax, nva_shard_accept) through the C ABI:
bit-exact against torch's argmax (the reference's sampler.py:66) on tie-heavy bf16 logits, against the numpy
restatement of the keys, against the reference's verify_drafts golden vectors, and at full Qwen3-8B vocabulary
size (151936) split over 1/2/4/8 shards."""
import numpy as np
import pytest
import torch

from oracle import argmax as am
from conftest import load_golden
from test_shard_argmax import _tricky_logits

pytestmark = pytest.mark.gpu
ACCEPT = load_golden("accept_golden.npz")


def _keys(logits, tp):
    from nvattn import ops
    shard = logits.shape[1] // tp
    return torch.stack([ops.shard_argmax(logits[:, r * shard:(r + 1) * shard], r * shard) for r in range(tp)])


@pytest.mark.parametrize("rows,vocab", [(1, 7), (5, 999), (24, 4096), (300, 37984)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_shard_argmax_keys_match_oracle(cuda, rows, vocab, dtype):
    from nvattn import ops
    x = _tricky_logits(rows, vocab, rows + vocab)
    keys = ops.shard_argmax(x.to(dtype).cuda(), 1000)
    ref = am.shard_argmax_keys(x.numpy(), 1000)
    assert np.array_equal(keys.cpu().numpy().view(np.uint64), ref)


def test_shard_argmax_strided_rows(cuda):
    """A column slice (row stride > width, not 16-byte aligned): the scalar path."""
    from nvattn import ops
    x = _tricky_logits(9, 1001, 3).to(torch.bfloat16).cuda()
    keys = ops.shard_argmax(x[:, 3:1000], 0)
    assert np.array_equal(keys.cpu().numpy().view(np.uint64), am.shard_argmax_keys(x[:, 3:1000].float().cpu().numpy(), 0))


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_full_vocab_greedy_equals_torch_argmax(cuda, tp):
    """510 rows (102 sequences x (1+4), the largest k=4 verify) of 151936 bf16 logits: k=0 accept = argmax."""
    from nvattn import ops
    g = torch.Generator(device=cuda).manual_seed(tp)
    x = (torch.randn(510, 151936, generator=g, device=cuda) * 1.3).to(torch.bfloat16)
    x[::17, 5000] = x[::17].max(dim=1).values      # ties with an earlier maximum in some rows
    keys = _keys(x, tp).view(tp, 510, 1)
    empty = torch.empty(510, 0, dtype=torch.int64, device=cuda)
    acc, nxt = ops.shard_accept(keys, empty, torch.zeros(510, dtype=torch.int64, device=cuda))
    assert torch.equal(nxt, x.argmax(dim=-1)) and int(acc.abs().sum()) == 0


@pytest.mark.parametrize("case", sorted(ACCEPT))
@pytest.mark.parametrize("tp", [1, 2, 4])
@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_shard_accept_matches_reference_golden(cuda, case, tp, dtype):
    from nvattn import ops
    c = ACCEPT[case]
    t = torch.from_numpy(c["target"]).long()
    S, K1 = t.shape
    vocab = (int(t.max()) // (8 * tp) + 1) * 8 * tp
    logits = torch.zeros(S * K1, vocab, dtype=torch.bfloat16, device=cuda)
    logits.scatter_(1, t.reshape(-1, 1).cuda(), 1.0)
    keys = _keys(logits, tp).view(tp, S, K1)
    d = torch.from_numpy(c["drafts"]).reshape(S, K1 - 1).to(dtype).cuda()
    acc, nxt = ops.shard_accept(keys, d, torch.from_numpy(c["num_drafts"]).to(dtype).cuda())
    assert acc.dtype == nxt.dtype == dtype
    assert acc.cpu().tolist() == c["num_accepted"].tolist() and nxt.cpu().tolist() == c["next_token"].tolist()


@pytest.mark.parametrize("k", [1, 2, 4, 8])
def test_shard_accept_config3_equals_verify_drafts_greedy(cuda, k):
    """Config 3's accept inputs as logits (random bf16 logits whose argmax is the target id with draft match
    probability 0.7), split over 2 shards: same result as the unsharded argmax + greedy accept kernel."""
    from nvattn import ops
    from nvattn.sampler import verify_drafts_greedy
    S, V = 512 // (1 + k), 151936
    g = torch.Generator(device=cuda).manual_seed(k)
    logits = (torch.randn(S * (k + 1), V, generator=g, device=cuda)).to(torch.bfloat16)
    top = logits.argmax(dim=-1).view(S, k + 1)
    match = torch.rand(S, k, generator=g, device=cuda) < 0.7
    drafts = torch.where(match, top[:, :k], (top[:, :k] + 1) % V)
    nd = torch.randint(0, k + 1, (S,), generator=g, device=cuda)
    ra, rn = verify_drafts_greedy(logits, drafts, nd)
    acc, nxt = ops.shard_accept(_keys(logits, 2).view(2, S, k + 1), drafts, nd)
    assert torch.equal(acc, ra) and torch.equal(nxt, rn)
