"""Decode-layer step (BASELINE config 5 and smaller) vs the numpy restatement of the
reference's full_decode_np (examples/qwen_megakernel.py:320-342).  bf16 storage with
fp32 accumulation: max-abs <= 2e-2 and relative Frobenius <= 5e-3 on the output."""
import numpy as np
import pytest

from oracle import numerics as orc

pytestmark = pytest.mark.gpu


def _run(cfg, seed=0):
    import torch
    from enigma.decode_layer import DecodeLayer
    layer = DecodeLayer.random(cfg, seed=seed)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    x = torch.randn(cfg.batch, cfg.hidden, device="cuda", generator=g).bfloat16()
    kc0 = layer.k_cache.float().cpu().numpy()
    vc0 = layer.v_cache.float().cpu().numpy()
    out = layer.step(x)
    torch.cuda.synchronize()
    w = {k: v.float().cpu().numpy() for k, v in layer.w.items()}
    ref, q, k, v = orc.decode_layer(x.float().cpu().numpy(), w, kc0, vc0, layer._cos.cpu().numpy(),
                                    layer._sin.cpu().numpy(), cfg.cache_len, cfg.heads_q,
                                    cfg.heads_kv, cfg.head_dim, cfg.eps)
    return layer, out.float().cpu().numpy(), ref, k, v


@pytest.mark.parametrize("batch,hidden,hq,hkv,inter,cache,cap", [
    (2, 128, 2, 1, 256, 10, 74), (64, 896, 14, 2, 4864, 2048, 2112), (5, 512, 8, 2, 1024, 300, 364),
    (1, 1024, 16, 8, 3072, 32, 96),
    (4, 128, 2, 1, 96, 10, 74),          # intermediate a multiple of 32, not of 64
    (128, 256, 4, 2, 512, 200, 264),     # the largest batch: a full 128-row A box
    (3, 256, 4, 1, 512, 299, 300),       # the appended key in the cache's last slot
    (24, 256, 4, 2, 512, 600, 640)])     # 48 units: clusters of 4 CTAs per unit
def test_decode_layer(cuda, batch, hidden, hq, hkv, inter, cache, cap):
    from enigma.decode_layer import DecodeConfig
    cfg = DecodeConfig(batch=batch, hidden=hidden, heads_q=hq, heads_kv=hkv, intermediate=inter,
                       cache_len=cache, cache_capacity=cap)
    layer, got, ref, k_new, v_new = _run(cfg)
    assert orc.max_abs(got, ref) <= 2e-2, orc.max_abs(got, ref)
    assert orc.rel_fro(got, ref) <= 5e-3, orc.rel_fro(got, ref)
    kc = layer.k_cache[:, :, cache].float().cpu().numpy()
    vc = layer.v_cache[:, :, cache].float().cpu().numpy()
    assert orc.rel_fro(kc, k_new) <= 5e-3 and orc.rel_fro(vc, v_new) <= 5e-3


@pytest.mark.parametrize("batch,hkv,cache,cap", [
    (3, 2, 40, 64),        # 6 units: flat-range attention, global-memory merge
    (64, 2, 300, 320)])    # 128 units: 2-CTA clusters per unit, DSMEM merge
def test_decode_advance_two_tokens(cuda, batch, hkv, cache, cap):
    """Two steps with advance=True: the second attends over the first step's appended k/v."""
    import torch
    from enigma.decode_layer import DecodeConfig, DecodeLayer, rope_tables
    cfg = DecodeConfig(batch=batch, hidden=256, heads_q=4, heads_kv=hkv, intermediate=512,
                       cache_len=cache, cache_capacity=cap)
    layer = DecodeLayer.random(cfg, seed=3)
    x1 = torch.randn(batch, 256, device="cuda").bfloat16()
    x2 = torch.randn(batch, 256, device="cuda").bfloat16()
    layer.step(x1, advance=True)
    kc = layer.k_cache.float().cpu().numpy()
    vc = layer.v_cache.float().cpu().numpy()
    out = layer.step(x2).float().cpu().numpy()
    c, s = rope_tables(cfg, cache + 1)
    w = {k: v.float().cpu().numpy() for k, v in layer.w.items()}
    ref = orc.decode_layer(x2.float().cpu().numpy(), w, kc, vc, c, s, cache + 1, 4, hkv, 64,
                           cfg.eps)[0]
    assert orc.rel_fro(out, ref) <= 5e-3


def test_decode_rejects_bad_desc(cuda):
    from enigma import _native
    from enigma.decode_layer import DecodeConfig, DecodeLayer
    layer = DecodeLayer.random(DecodeConfig(batch=2, hidden=128, heads_q=2, heads_kv=1,
                                            intermediate=256, cache_len=8, cache_capacity=16))
    layer.desc.head_dim = 128
    with pytest.raises(_native.EnigmaCudaError, match="head_dim must be 64"):
        layer.step(__import__("torch").zeros(2, 128, device="cuda").bfloat16())


@pytest.mark.parametrize("batch,hkv", [(8, 1), (64, 2)])
def test_decode_graph_replay_matches(cuda, batch, hkv):
    """A replayed CUDA graph gives the eager step's bits (every reduction has a fixed order)."""
    import torch
    from enigma.decode_layer import DecodeConfig, DecodeLayer
    layer = DecodeLayer.random(DecodeConfig(batch=batch, hidden=256, heads_q=4, heads_kv=hkv,
                                            intermediate=512, cache_len=300, cache_capacity=320))
    x = torch.randn(batch, 256, device="cuda").bfloat16()
    eager = layer.step(x).float().cpu().numpy()
    out = torch.empty_like(x)
    replay = layer.capture(x, out)
    replay()
    torch.cuda.synchronize()
    assert orc.max_abs(out.float().cpu().numpy(), eager) == 0.0
