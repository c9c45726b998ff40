"""Sharded operators on the GPU with a one-rank NCCL group: the shard + all-gather path
returns what the unsharded operator returns."""
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nccl_group(cuda):
    import torch.distributed as dist
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    if not dist.is_initialized():
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0,
                                world_size=1)
    yield
    dist.destroy_process_group()


def test_sharded_ops_match(nccl_group):
    import torch
    from enigma import cuda_ops, shard
    x = torch.randn(1000, 2048, device="cuda").bfloat16()
    w = torch.ones(2048, device="cuda").bfloat16()
    assert torch.equal(shard.rmsnorm_rows(x, w, gather=True), cuda_ops.rmsnorm(x, w))
    a = torch.randn(300, 256, device="cuda").bfloat16()
    b = torch.randn(256, 512, device="cuda").bfloat16()
    assert torch.equal(shard.gemm_mblocks(a, b, gather=True), cuda_ops.gemm(a, b))
    q = torch.randn(2, 4, 256, 128, device="cuda").bfloat16()
    k = torch.randn(2, 2, 256, 128, device="cuda").bfloat16()
    v = torch.randn(2, 2, 256, 128, device="cuda").bfloat16()
    got = shard.sdpa_heads(q, k, v, causal=True, gather=True)
    assert torch.equal(got, cuda_ops.sdpa(q, k, v, causal=True))


def test_decode_sequences_one_rank_matches_layer(nccl_group):
    """decode_sequences with one rank: the rank holds the whole batch, and gathering its
    output gives the layer's own step (same kernels, same inputs: bit-identical)."""
    import torch
    from enigma import shard
    from enigma.decode_layer import DecodeConfig, DecodeLayer
    full = DecodeConfig(batch=8, hidden=256, heads_q=4, heads_kv=2, intermediate=512,
                        cache_len=100, cache_capacity=128)
    cfg = shard.decode_shard_config(full)
    assert cfg.batch == 8
    a = DecodeLayer.random(cfg, seed=3)
    b = DecodeLayer.random(full, seed=3)
    x = torch.randn(8, 256, device="cuda").bfloat16()
    got = shard.decode_sequences(a, x, gather=True)
    assert torch.equal(got, b.step(x))
