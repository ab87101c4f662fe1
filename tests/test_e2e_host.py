"""Host-side pieces of the config-5 end-to-end harness (nvattn/e2e.py) that need no GPU: the request set, the
same-shape warm-up requests the bench's e2e rows use, and that bench.py asks for that warm-up in both arms."""
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "nano-vllm-spec-decode_b200")
if PKG not in sys.path:
    sys.path.insert(0, PKG)

from nvattn import e2e  # noqa: E402


def test_config5_prompts_shape_and_repeated_span():
    prompts = e2e.config5_prompts(64, 1024, seed=0)
    assert len(prompts) == 64 and all(len(p) == 1024 for p in prompts)
    assert all(0 <= t < 151643 for p in prompts for t in p)   # below Qwen3's special tokens
    for p in prompts:
        tail = p[1024 - 4 * 128:]
        assert tail == tail[:128] * 4   # one 128-token span repeated 4 times: n-gram lookups match from step one
    assert prompts == e2e.config5_prompts(64, 1024, seed=0)   # seeded


def test_shape_warmup_requests_share_no_cache_block_with_measured_ones():
    """The warm-up requests (prompt seed + 1) have the measured shape but share no 256-token prefix block with the
    measured requests, so the timed run gets no prefix-cache hits from the warm-up."""
    measured = e2e.config5_prompts(64, 1024, seed=0)
    warm = e2e.config5_prompts(64, 1024, seed=1)
    assert len(warm) == len(measured) and {len(p) for p in warm} == {1024}
    for blocks in (1, 2, 3, 4):
        m = {tuple(p[:256 * blocks]) for p in measured}
        assert not any(tuple(p[:256 * blocks]) in m for p in warm)


def test_bench_e2e_rows_ask_for_the_shape_warmup():
    with open(os.path.join(REPO, "bench.py")) as f:
        src = f.read()
    assert '"--shape-warmup"' in src
    import inspect
    assert "shape_warmup" in inspect.signature(e2e.run_arm).parameters
