"""GPU parity of the fused attention prologue nva_qk_norm_rope_store (q / k RMSNorm + rotary + KV scatter in one
kernel) through the C ABI: q and k against the reference's own RMSNorm / rotary layers (golden vectors) within
bf16 rounding (the reduction order of the mean and rsqrt differ; at least 99% of the values are bit-identical), and
the scatter bit-exact: the cache rows at the slots hold exactly the kernel's k and the input v, slot -1 writes
nothing, an out-of-range slot writes nothing and sets bit 1 of the device error word."""
import pytest
import torch

from oracle import prologue
from conftest import load_golden
from test_prologue_oracle import case_inputs, bf16

pytestmark = pytest.mark.gpu
GOLD = load_golden("prologue_golden.npz")


def _close(got, ref, what):
    got, ref = got.float().cpu(), ref.float().cpu()
    err = (got - ref).abs()
    assert bool((err <= 2e-2 + 1e-2 * ref.abs()).all()), f"{what}: max err {float(err.max()):.4g}"
    same = float((got == ref).float().mean())
    assert same >= 0.99, f"{what}: only {same:.4f} bit-identical"


@pytest.mark.parametrize("case", sorted(GOLD))
def test_prologue_matches_reference_layers_and_scatters(cuda, case):
    from nvattn import ops, _lib
    c = GOLD[case]
    T, H, KVH, table, qkv, pos, qw, kw = case_inputs(c)
    nb = 4
    kc = torch.zeros(nb, 256, KVH, 128, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    g = torch.Generator().manual_seed(T)
    slots = torch.randperm(nb * 256, generator=g)[:T].to(torch.int32)
    slots[::5] = -1
    _lib.clear_device_error()
    q, k, v = ops.qk_norm_rope_store(qkv.cuda(), pos.cuda(), table.cuda(), qw.cuda(), kw.cuda(), 1e-6, H, KVH,
                                     kc, vc, slots.cuda(), want_k=True)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    _close(q, bf16(c["q"]).view(T, H, 128), f"{case} q")
    _close(k, bf16(c["k"]).view(T, KVH, 128), f"{case} k")
    live = slots >= 0
    kf, vf = kc.view(-1, KVH, 128).cpu(), vc.view(-1, KVH, 128).cpu()
    assert torch.equal(kf[slots[live].long()], k.cpu()[live])
    assert torch.equal(vf[slots[live].long()], v.cpu()[live])
    untouched = torch.ones(nb * 256, dtype=torch.bool)
    untouched[slots[live].long()] = False
    assert kf[untouched].abs().sum() == 0 and vf[untouched].abs().sum() == 0


def test_prologue_without_cache_and_bad_slot(cuda):
    """No cache (the piecewise pre_attn form): q and k only.  Then an out-of-range slot: skipped, error bit set."""
    from nvattn import ops, _lib
    c = GOLD["qwen3_8b_decode"]
    T, H, KVH, table, qkv, pos, qw, kw = case_inputs(c)
    q, k, _ = ops.qk_norm_rope_store(qkv.cuda(), pos.cuda(), table.cuda(), qw.cuda(), kw.cuda(), 1e-6, H, KVH,
                                     want_k=True)
    rq, rk, _ = prologue.qk_prologue_ref(qkv, pos, table, qw, kw, 1e-6, H, KVH)
    _close(q, rq, "q (no cache)")
    _close(k, rk, "k (no cache)")
    kc = torch.zeros(1, 256, KVH, 128, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    slots = torch.full((T,), -1, dtype=torch.int32)
    slots[3] = 256                      # one past the pool
    _lib.clear_device_error()
    ops.qk_norm_rope_store(qkv.cuda(), pos.cuda(), table.cuda(), qw.cuda(), kw.cuda(), 1e-6, H, KVH, kc, vc,
                           slots.cuda())
    assert _lib.device_error() & 1
    assert kc.abs().sum() == 0 and vc.abs().sum() == 0
    _lib.clear_device_error()
