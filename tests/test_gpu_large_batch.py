"""GPU parity at the benchmarked batch sizes (B = 256, 257, 448 rows; H=128, P=80, N=128, fp8
cold, c=4) against the CPU oracle on a sample of rows.

FLUSH counts and numbers the batch's flushing rows before splitting their items over the grid
(the tensor-core FLUSH: each of 128 threads takes a contiguous block of up to 8 rows and a
block-wide scan numbers them; the banded FLUSH of other configurations: passes of 256 rows);
a row past 256 is numbered from the rows before it, and that number decides which CTA
replays it.  Rows are independent, so the oracle only has to follow a sample of them (rows 0,
1, 255, 256, 257, 300, 447 where they exist and 32 random ones): before every step the
oracle's copy of those rows is re-synced from the GPU pool, the whole batch steps on the GPU,
the sampled rows step in the oracle, and y and the sampled pool rows are compared at the
per-step bar.  Lockstep prompts (every row flushes on the same token) and per-slot phases
(every token a quarter of the rows flushes), a permuted slot map and padded rows.

The last test replays the benchmark's own 27-layer CUDA graph (bench.py ``Workload``, B=448)
once and checks sampled rows of three layers against the oracle run over the same 4 tokens.
Reference semantics: scale/vllm_v4_patch.py:140-179 (decode_readout), scale/v4_fused_decode.py:76-92
(flush replay).
"""
import math

import pytest
import torch

import oracle as O
from tests import _helpers as Hh

pytestmark = pytest.mark.gpu

H, P, N, G, PB, C = 128, 80, 128, 8, 32, 4
FIXED_ROWS = (0, 1, 255, 256, 257, 300, 447)


def _sample_rows(b, gen, extra=32):
    fixed = [r for r in FIXED_ROWS if r < b]
    rest = torch.tensor([r for r in torch.randperm(b, generator=gen).tolist() if r not in fixed][:extra])
    return torch.cat([torch.tensor(fixed), rest]).long()


class SampledOracle:
    """Oracle pool holding only the sampled slots: oracle slot i <-> GPU slot gslots[i]."""

    def __init__(self, gslots, c=C):
        self.gslots = gslots.long()
        self.pool = O.TieredPoolRef(len(gslots), H, P, N, G, PB, c, O.FP8, torch.bfloat16)

    def sync_from(self, gpool, layer=0):
        s, o = self.gslots.cuda(), self.pool
        o.hot.copy_(gpool.hot[layer][s].cpu())
        o.cold.copy_(gpool.cold[layer][s].cpu())
        o.scale.copy_(gpool.scale[layer][s].cpu())
        o.glog.copy_(gpool.glog[layer][s].cpu())
        o.t.copy_(gpool.t[layer][s][:, 0].cpu())
        o.ring_x.copy_(gpool.ring_x[layer][s].cpu())
        o.ring_dt.copy_(gpool.ring_dt[layer][s][..., :o.c].cpu())
        o.ring_b.copy_(gpool.ring_b[layer][s].cpu())

    def compare(self, gpool, layer=0, per_step=True, budget=None):
        """Per-step bar (identical state before the step): hot to fp32 reassociation, t exact,
        glog to 1e-6, fp8 codes within 1 ulp and at most 1e-4 of them differing, scales to
        1e-5.  Free-running (per_step=False): cold within the accumulated one-ulp budget."""
        s, o = self.gslots.cuda(), self.pool
        torch.testing.assert_close(gpool.hot[layer][s].cpu(), o.hot, rtol=1e-5, atol=1e-6)
        assert torch.equal(gpool.t[layer][s].cpu(), o.t[:, None].expand(-1, H).to(torch.int32))
        torch.testing.assert_close(gpool.glog[layer][s].cpu(), o.glog, rtol=1e-6, atol=1e-6)
        gc = gpool.cold[layer][s].cpu()
        if per_step:
            d = Hh.fp8_ulp_dist(gc, o.cold)
            assert int(d.max()) <= 1, f"fp8 cold differs by up to {int(d.max())} ulp"
            assert float((d > 0).float().mean()) <= 1e-4
            torch.testing.assert_close(gpool.scale[layer][s].cpu(), o.scale, rtol=1e-5, atol=0)
            return None
        gv = O.dequantize_rows(gc, gpool.scale[layer][s].cpu())
        ov = O.dequantize_rows(o.cold, o.scale)
        amax = ov.abs().amax(dim=-1, keepdim=True)
        per = 0.13 * ov.abs() + 2e-3 * amax + 1e-7
        budget = per if budget is None else budget + per
        worst = float(((gv - ov).abs() / budget).max())
        assert worst <= 1.0, f"cold off by {worst:.2f}x the accumulated one-ulp budget"
        return budget


def _prefill_random(gpool, S, seed, layer=0):
    from nested_ssm_b200 import prefill_split
    g = torch.Generator(device="cuda").manual_seed(seed)
    for s0 in range(0, S, 64):
        sl = torch.arange(s0, min(S, s0 + 64), dtype=torch.int32, device="cuda")
        st = torch.randn(sl.numel(), H, P, N, device="cuda", generator=g) * math.sqrt(0.1)
        prefill_split(gpool, layer, st, sl)
    torch.cuda.synchronize()


@pytest.mark.parametrize("phases", ["lockstep", "per_slot"])
@pytest.mark.parametrize("b", [256, 257, 448])
def test_benchmarked_batch_sampled_rows(b, phases):
    from nested_ssm_b200 import TieredSlotPool, tiered_state_update
    gen = torch.Generator().manual_seed(1000 + b)
    S = b + 40
    slot_of_row = torch.randperm(S, generator=gen)[:b]            # permuted slot map
    gpool = TieredSlotPool(1, S, H, P, N, G, PB, C, "fp8", torch.bfloat16, "cuda", max_batch=b)
    _prefill_random(gpool, S, seed=b)
    if phases == "per_slot":   # each slot starts at its own token count mod c
        gpool.t[0] = (torch.arange(S, device="cuda", dtype=torch.int32) % C)[:, None]
    rows = _sample_rows(b, gen)
    orc = SampledOracle(slot_of_row[rows])
    prm = O.make_params(H, G, N, seed=b)[0]
    steps = 2 * C + 1
    xs, dts, Bs, Cs = O.make_inputs(b, H, P, G, N, steps, seed=b)
    A, D, dtb = prm["A"].cuda(), prm["D"].cuda(), prm["dt_bias"].cuda()
    flushed_rows_seen = 0
    for s in range(steps):
        pad = torch.rand(b, generator=gen) < 0.05
        pad[rows[s % len(rows)]] = True                           # a sampled row padded each step
        slots = torch.where(pad, torch.full_like(slot_of_row, -1), slot_of_row)
        Br = O.rot_flat(Bs[s].reshape(b, G * N), prm["R"]).reshape(b, G, N)
        Cr = O.rot_flat(Cs[s].reshape(b, G * N), prm["R"]).reshape(b, G, N)
        orc.sync_from(gpool)
        t_before = gpool.t[0][slot_of_row.cuda(), 0].cpu()
        out = torch.zeros(b, H, P, device="cuda")
        tiered_state_update(gpool, 0, xs[s].cuda(), dts[s].cuda(), A, Br.cuda(), Cr.cuda(), D, dtb, True,
                            slots.to(torch.int32).cuda(), -1, out, None, 1e-3)
        osl = torch.where(pad[rows], torch.full((len(rows),), -1), torch.arange(len(rows)))
        yo = O.tiered_step(orc.pool, osl, xs[s][rows], dts[s][rows], Br[rows], Cr[rows], prm["A"], prm["D"],
                           prm["dt_bias"], 1e-3)
        torch.cuda.synchronize()
        yg = out.cpu()
        Hh.assert_y_close(yg[rows], yo, f"B={b} {phases} step {s}")
        assert torch.all(yg[pad] == 0), "padded rows must be left untouched"
        orc.compare(gpool)
        # rows past 256 at a chunk boundary on this token: FLUSH's later counting passes ran
        fl = (~pad) & ((t_before + 1) % C == 0)
        flushed_rows_seen += int(fl[256:].sum()) if b > 256 else 0
    if b > 256:
        assert flushed_rows_seen > 0
    assert int(gpool.status.item()) == 0


def test_bench_graph_replay_sampled_rows():
    """One replay of the benchmark's 27-layer CUDA graph (4 tokens from a chunk start; the
    4th flushes every slot) at B=448 against the oracle on sampled rows of layers 0, 13 and
    26, free-running over the 4 tokens from the state before the replay.  The last token's y
    is read before its flush, so it is held to the per-step y bar plus the rounding of the
    benchmark's bf16 output (2^-8 relative); hot state to fp32 reassociation; the flushed cold codes within
    one fp8 ulp (the GPU's and the CPU's softplus may differ by an fp32 ulp in dt between
    syncs, which can move a code by one step) and rarely different at all."""
    import argparse
    import bench
    from nested_ssm_b200 import rot_flat
    args = argparse.Namespace(layers=27, batch=448, hot=PB, chunk=C, cold="fp8")
    wl = bench.Workload(args, rank=0)
    NI = bench.Workload.NI
    assert NI == C
    g = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g, stream=cap):
            for k in range(NI):
                wl.step(1 + k)
    torch.cuda.current_stream().wait_stream(cap)
    torch.cuda.synchronize()
    gen = torch.Generator().manual_seed(7)
    rows = _sample_rows(448, gen, extra=16)
    layers = (0, 13, 26)
    orcs = {}
    for l in layers:
        orcs[l] = SampledOracle(wl.slots[rows.cuda()].cpu())
        orcs[l].sync_from(wl.pool, l)
    B = wl.B
    yo = {}
    for k in range(NI):
        i = (1 + k) % NI
        for l in layers:
            BCr = rot_flat(wl.BC[i, l], wl.R[l]).cpu()          # the rotation the graph computes
            Br = BCr[:B].view(B, G, N)[rows]
            Cr = BCr[B:].view(B, G, N)[rows]
            yo[l] = O.tiered_step(orcs[l].pool, torch.arange(len(rows)), wl.x[i, l][rows.cuda()].cpu(),
                                  wl.dt[i, l][rows.cuda()].cpu(), Br, Cr, wl.A[l].cpu(), wl.D[l].cpu(),
                                  wl.dtb[l].cpu(), 1e-3)
    g.replay()
    torch.cuda.synchronize()
    for l in layers:
        o = orcs[l].pool
        assert int(o.t[0]) == NI and float(o.glog.abs().max()) == 0.0   # every sampled slot flushed
        # the benchmark's y is bf16: its rounding adds up to 2^-8 relative to the y bar
        torch.testing.assert_close(wl.y[l][rows.cuda()].float().cpu(), yo[l], rtol=Hh.Y_RTOL + 2.0 ** -8,
                                   atol=Hh.Y_ATOL, msg=lambda m: f"layer {l}: {m}")
        orcs[l].compare(wl.pool, l, per_step=False)
        d = Hh.fp8_ulp_dist(wl.pool.cold[l][orcs[l].gslots.cuda()].cpu(), o.cold)
        assert int(d.max()) <= 1 and float((d > 0).float().mean()) <= 1e-3, f"layer {l}: cold codes"
    wl.pool.check_status()
    del g, wl
    torch.cuda.empty_cache()


@pytest.mark.parametrize("c", [16, 64])
def test_flush_with_full_random_ring(c):
    """The c = 16 / 64 FLUSH (the rank-c update on the tensor cores) with every ring entry
    random: the ring's x, dt and B' of all slots are filled with seeded values (B' bf16-exact,
    as the step writes it), the rows sit one to three tokens before their chunk boundary
    (staggered phases, some rows past their first chunk) and then step per token from
    identical state, so each token a third of the 96 rows replays a whole random ring."""
    from nested_ssm_b200 import TieredSlotPool, tiered_state_update
    b, S = 96, 100
    gen = torch.Generator().manual_seed(500 + c)
    slot_of_row = torch.randperm(S, generator=gen)[:b]
    gpool = TieredSlotPool(1, S, H, P, N, G, PB, c, "fp8", torch.bfloat16, "cuda", max_batch=b)
    _prefill_random(gpool, S, seed=c)
    g = torch.Generator(device="cuda").manual_seed(c)
    gpool.ring_x[0].copy_(torch.randn(gpool.ring_x[0].shape, device="cuda", generator=g).to(torch.bfloat16))
    gpool.ring_dt[0].copy_(torch.rand(gpool.ring_dt[0].shape, device="cuda", generator=g) * 0.2 + 1e-3)
    rb = (torch.randn(gpool.ring_b[0].shape, device="cuda", generator=g) / math.sqrt(N)).to(torch.bfloat16)
    gpool.ring_b[0].copy_(rb.float())
    rows = torch.arange(b)
    tstart = (c - 1 - rows % 3) + c * (rows % 2)              # 1-3 tokens before a boundary
    gpool.t[0][slot_of_row.cuda()] = tstart.to(torch.int32).cuda()[:, None]
    orc = SampledOracle(slot_of_row, c=c)
    prm = O.make_params(H, G, N, seed=c)[0]
    xs, dts, Bs, Cs = O.make_inputs(b, H, P, G, N, 3, seed=c)
    A, D, dtb = prm["A"].cuda(), prm["D"].cuda(), prm["dt_bias"].cuda()
    for s in range(3):
        Br = O.rot_flat(Bs[s].reshape(b, G * N), prm["R"]).reshape(b, G, N)
        Cr = O.rot_flat(Cs[s].reshape(b, G * N), prm["R"]).reshape(b, G, N)
        orc.sync_from(gpool)
        out = torch.zeros(b, H, P, device="cuda")
        tiered_state_update(gpool, 0, xs[s].cuda(), dts[s].cuda(), A, Br.cuda(), Cr.cuda(), D, dtb, True,
                            slot_of_row.to(torch.int32).cuda(), -1, out, None, 1e-3)
        yo = O.tiered_step(orc.pool, torch.arange(b), xs[s], dts[s], Br, Cr, prm["A"], prm["D"], prm["dt_bias"], 1e-3)
        torch.cuda.synchronize()
        Hh.assert_y_close(out.cpu(), yo, f"c={c} step {s}")
        assert int(((tstart + s + 1) % c == 0).sum()) == b // 3     # a third of the rows flushed
        orc.compare(gpool)
    assert int(gpool.status.item()) == 0
