"""The Qwen2 workload's fixed-shape decode step (a 0-d position tensor,
attention over the whole KV cache with later positions masked, as a CUDA
graph needs) gives the same logits as the sliced-cache step with a Python
position, on a tiny fp32 model on the CPU, over several steps."""
import torch

from vla_abft_estimate_b200.workloads import build_qwen2

TINY = dict(hidden=64, inter=128, layers=2, heads=4, kv_heads=2, head_dim=16, vocab=100, rope_theta=10000.0,
            eps=1e-6)


def test_tensor_position_decode_matches_sliced_cache_decode():
    model = build_qwen2(TINY, "cpu", seed=0, dtype=torch.float32)
    ids = torch.randint(0, TINY["vocab"], (7,), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        c_int, c_tensor = model.new_caches(16), model.new_caches(16)
        p_int = model(ids, c_int, 0)
        p_tensor = model(ids, c_tensor, 0)
        assert torch.equal(p_int, p_tensor)
        pos = torch.tensor(7)
        tok = ids[-1:]
        for i in range(4):
            a = model(tok, c_int, 7 + i)
            b = model(tok, c_tensor, pos)
            pos += 1
            assert torch.allclose(a, b, atol=1e-5, rtol=1e-5), f"step {i}"
            for x, y in zip(c_int, c_tensor):
                assert torch.allclose(x[:, :, : 8 + i], y[:, :, : 8 + i], atol=1e-6)
            tok = a[-1:].argmax(-1)
    assert int(pos) == 11
