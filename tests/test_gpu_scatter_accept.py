"""GPU parity of the integer / byte kernels: KV scatter and greedy accept length, bit-exact against the golden
vectors of the reference and against the C oracle at full BASELINE sizes."""
import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden
from test_oracle import _scatter_inputs, _tensor

pytestmark = pytest.mark.gpu

SCATTER = load_golden("scatter_golden.npz")
ACCEPT = load_golden("accept_golden.npz")


@pytest.mark.parametrize("case", sorted(SCATTER))
def test_scatter_matches_reference_golden(cuda, case):
    from nvattn import ops
    c = SCATTER[case]
    key, value, kc, vc, slots, dt = _scatter_inputs(c)
    # rebuild the strided views on the device (same strides as the reference's inputs)
    kb = key._base if key._base is not None else key
    vb = value._base if value._base is not None else value
    kd = kb.cuda().as_strided(key.shape, key.stride(), key.storage_offset())
    vd = vb.cuda().as_strided(value.shape, value.stride(), value.storage_offset())
    kcd, vcd = kc.cuda(), vc.cuda()
    ops.store_kvcache(kd, vd, kcd, vcd, slots.cuda())
    torch.cuda.synchronize()
    assert torch.equal(kcd.cpu(), _tensor(c["k_out"], dt).view(kc.shape))
    assert torch.equal(vcd.cpu(), _tensor(c["v_out"], dt).view(vc.shape))


@pytest.mark.parametrize("n_tokens,num_blocks", [(64, 2048), (2048, 256), (1, 4)])
def test_scatter_full_size_matches_c_oracle(cuda, n_tokens, num_blocks):
    from nvattn import ops
    g = torch.Generator().manual_seed(n_tokens)
    KVH, D = 8, 128
    qkv = torch.randn(n_tokens, (32 + 16) * D, generator=g).to(torch.bfloat16)   # k, v are column slices
    key = qkv[:, 32 * D:40 * D].view(n_tokens, KVH, D)
    value = qkv[:, 40 * D:48 * D].view(n_tokens, KVH, D)
    slots = torch.randperm(num_blocks * 256, generator=g)[:n_tokens].to(torch.int32)
    slots[::7] = -1
    kc = torch.zeros(num_blocks, 256, KVH, D, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    oracle.store_kvcache(key, value, kc, vc, slots)
    qkv_d = qkv.cuda()
    kd = qkv_d[:, 32 * D:40 * D].view(n_tokens, KVH, D)
    vd = qkv_d[:, 40 * D:48 * D].view(n_tokens, KVH, D)
    kcd = torch.zeros_like(kc, device=cuda)
    vcd = torch.zeros_like(vc, device=cuda)
    ops.store_kvcache(kd, vd, kcd, vcd, slots.cuda())
    assert torch.equal(kcd.cpu(), kc) and torch.equal(vcd.cpu(), vc)


def test_scatter_out_of_range_slot_sets_error_and_writes_nothing(cuda):
    from nvattn import ops, _lib
    _lib.clear_device_error()
    key = torch.randn(2, 8, 128, device=cuda).to(torch.bfloat16)
    kc = torch.zeros(1, 256, 8, 128, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    ops.store_kvcache(key, key, kc, vc, torch.tensor([256, 3], dtype=torch.int32, device=cuda))
    assert _lib.device_error() & 1
    assert torch.equal(kc[0, 3], key[1]) and kc.view(-1, 8, 128)[:3].abs().sum() == 0
    _lib.clear_device_error()


@pytest.mark.parametrize("case", sorted(ACCEPT))
@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_accept_matches_reference_golden(cuda, case, dtype):
    from nvattn import ops
    c = ACCEPT[case]
    t = torch.from_numpy(c["target"]).to(dtype).cuda()
    S, K1 = t.shape
    d = torch.from_numpy(c["drafts"]).to(dtype).reshape(S, K1 - 1).cuda()
    nd = torch.from_numpy(c["num_drafts"]).to(dtype).cuda()
    a, n = ops.greedy_accept(t, d, nd)
    assert a.cpu().tolist() == c["num_accepted"].tolist()
    assert n.cpu().tolist() == c["next_token"].tolist()


@pytest.mark.parametrize("case", sorted(ACCEPT))
def test_verify_drafts_greedy_matches_reference_golden(cuda, case):
    """The golden cases came from the reference's verify_drafts fed one-hot logits whose argmax is the target id;
    the same logits (bf16, as the LM head gives them) go through nvattn.sampler.verify_drafts_greedy."""
    from nvattn.sampler import verify_drafts_greedy
    c = ACCEPT[case]
    t = torch.from_numpy(c["target"]).cuda()
    S, K1 = t.shape
    logits = torch.zeros(S * K1, max(int(t.max()) + 1, 2), dtype=torch.bfloat16, device=cuda)
    logits.scatter_(1, t.reshape(-1, 1), 1.0)
    d = torch.from_numpy(c["drafts"]).reshape(S, K1 - 1).cuda()
    a, n = verify_drafts_greedy(logits, d, torch.from_numpy(c["num_drafts"]).cuda())
    assert a.dtype == n.dtype == torch.int64
    assert a.cpu().tolist() == c["num_accepted"].tolist()
    assert n.cpu().tolist() == c["next_token"].tolist()


@pytest.mark.parametrize("k", [1, 2, 4, 8])
def test_accept_config3_large_batch(cuda, k):
    """Config 3 shape at 512 // (1+k) sequences (the largest verify batch, config.py:69-73)."""
    from nvattn import ops
    from nvattn.workloads import accept_config
    S = 512 // (1 + k)
    t, d, nd = accept_config(k, S=S, seed=100 + k)
    nd = torch.randint(0, k + 1, (S,), generator=torch.Generator().manual_seed(k)).to(torch.int32)
    ra, rn = oracle.greedy_accept(t.numpy(), d.numpy(), nd.numpy())
    a, n = ops.greedy_accept(t.cuda(), d.cuda(), nd.cuda())
    assert np.array_equal(a.cpu().numpy(), ra) and np.array_equal(n.cpu().numpy(), rn)
