"""The decode step captured in a CUDA graph and replayed gives the same bits as eager launches.

Two layers share one rotation workspace (as a decode loop does): layer l + 1's rotation
overwrites the rotated B, C that layer l's tiered update read, and every layer's FLUSH
decides from the token counts its STEP wrote whether a slot is at a chunk boundary, so a
graph replayed across two chunks must flush on the same tokens as the eager loop.  This is
how bench.py runs the decode step.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

H, P, N, G = 128, 80, 128, 8


def _setup(L, B, c, seed):
    from nested_ssm_b200 import TieredSlotPool, prefill_split
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    pools = [TieredSlotPool(L, B + 8, H, P, N, G, 32, c, "fp8", torch.bfloat16, dev, max_batch=B) for _ in range(2)]
    slots = torch.randperm(B + 8, device=dev, generator=gen)[:B].to(torch.int32)
    slots[3] = -1
    for l in range(L):
        st = torch.randn(B, H, P, N, device=dev, generator=gen) * math.sqrt(0.1)
        for pool in pools:
            prefill_split(pool, l, st, slots)
    prm = dict(
        A=[-torch.exp(torch.rand(H, device=dev, generator=gen) * math.log(16.0)) for _ in range(L)],
        D=[torch.randn(H, device=dev, generator=gen) for _ in range(L)],
        dtb=[torch.log(torch.expm1(torch.rand(H, device=dev, generator=gen) * 0.099 + 1e-3)) for _ in range(L)],
        R=[torch.linalg.qr(torch.randn(G, N, N, device=dev, generator=gen))[0].contiguous() for _ in range(L)])
    T = 2 * c
    inp = dict(
        x=torch.randn(T, L, B, H, P, device=dev, generator=gen).to(torch.bfloat16),
        dt=torch.randn(T, L, B, H, device=dev, generator=gen).to(torch.bfloat16),
        BC=(torch.randn(T, L, 2 * B, G * N, device=dev, generator=gen) / math.sqrt(N)).to(torch.bfloat16))
    return pools, slots, prm, inp


def _token(pool, slots, prm, inp, k, BCr, y, L, B):
    from nested_ssm_b200 import rot_flat, tiered_state_update
    for l in range(L):
        rot_flat(inp["BC"][k, l], prm["R"][l], out=BCr)
        tiered_state_update(pool, l, inp["x"][k, l], inp["dt"][k, l], prm["A"][l], BCr[:B].view(B, G, N),
                            BCr[B:].view(B, G, N), prm["D"][l], prm["dtb"][l], True, slots, -1, y[k, l], None, 1e-3)


def test_graph_replay_matches_eager():
    L, B, c = 2, 96, 4
    pools, slots, prm, inp = _setup(L, B, c, seed=7)
    T = 2 * c
    dev = torch.device("cuda")
    BCr = [torch.empty(2 * B, G * N, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    ys = [torch.zeros(T, L, B, H, P, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    # eager: 2c tokens (two flushes)
    for k in range(T):
        _token(pools[0], slots, prm, inp, k, BCr[0], ys[0], L, B)
    # graph: c tokens captured once, replayed twice with the second half's inputs copied in
    stage = {key: v[:c].clone() for key, v in inp.items()}
    y_g = torch.zeros(c, L, B, H, P, dtype=torch.bfloat16, device=dev)
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g, stream=cap):
            for k in range(c):
                _token(pools[1], slots, prm, stage, k, BCr[1], y_g, L, B)
    torch.cuda.current_stream().wait_stream(cap)
    for half in range(2):
        for key in stage:
            stage[key].copy_(inp[key][half * c:(half + 1) * c])
        g.replay()
        ys[1][half * c:(half + 1) * c].copy_(y_g)
    torch.cuda.synchronize()
    del g
    pad = slots.long() < 0
    assert torch.equal(ys[0], ys[1]), "y differs between graph replay and eager launches"
    assert int(ys[0][:, :, pad].float().abs().sum()) == 0
    a, b = pools
    for name in ("hot", "cold", "scale", "glog", "t", "ring_x", "ring_dt", "ring_b"):
        ta, tb = getattr(a, name), getattr(b, name)
        if ta.dtype == torch.float8_e4m3fn:
            ta, tb = ta.view(torch.uint8), tb.view(torch.uint8)
        assert torch.equal(ta, tb), f"pool {name} differs between graph replay and eager launches"
    assert int(a.t[0, slots[0].long(), 0]) == T
    a.check_status()
    b.check_status()
