"""The CPU oracle against the golden fixtures made by running the reference's own code
(tests/golden/make_golden.py).  This is what pins the oracle that the GPU tests use.

* native fp32: ``oracle.native_step`` reproduces ``_v4_decode`` bit for bit; the replay
  semantics the kernels implement (``oracle.tiered_step``, fp32 cold) agree to fp32
  reassociation in y and state through three flushes, in modes stale / corr / coldoff.
* vLLM fp8: ``oracle.quantize_rows`` / ``prefill_split`` reproduce ``prefill_snapshot``'s
  codes and scales bit for bit; ``oracle.native_step`` reproduces ``decode_readout``'s y,
  t, glog and flush snapshots bit for bit; the replay semantics agree bit for bit until
  the first flush (after it the fp8-only cold master drifts from the fp32 master by design).
* rotation: ``oracle.rot_flat`` reproduces ``rot_flat`` in both precisions bit for bit.
* conv: ``oracle.conv_step`` + ``conv_split`` + the replay state op reproduce ``_v4_decode``
  with a real conv1d and the reference's ActRotMask activation (SiLU + rotation) to fp32
  rounding, and leave the conv state the transformers cache holds.
"""
import torch

import oracle as O
from tests import _golden as GD

# fp32 reassociation between the replay and the native full-state update
REPLAY_ATOL = 2e-6


def test_rot_flat_matches_reference():
    d = GD.load("rot_flat.npz")
    x, R = GD.bf16(d["x"]), d["R"]
    assert torch.equal(O.rot_flat(x, R, "native").view(torch.int16), d["out_bf16"])
    assert torch.equal(O.rot_flat(x, R, "fp32"), d["out_fp32"].to(torch.bfloat16))
    assert torch.equal(O.rot_flat(x.float(), R, "fp32"), d["out_fp32"])


def _native_run(mode):
    d = GD.load("native_decode_fp32.npz")
    inp = GD.native_inputs(mode)
    GD.check_sums(d, inp, f"{mode}_")
    cfg = inp["cfg"]
    b, H, P, N, G, pb, c = (cfg[k] for k in ("b", "H", "P", "N", "G", "pb", "c"))
    return d, inp, b, H, P, N, G, pb, c


def test_native_step_bitexact_vs_v4_decode():
    d, inp, b, H, P, N, G, pb, c = _native_run("stale")
    npool = O.NativePoolRef(b, H, P, N, pb, c, torch.float32)
    slots = torch.arange(b)
    O.prefill_split(npool, slots, inp["s0"])
    for s in range(inp["steps"]):
        Br, Cr = GD.bf16(d["stale_Br"][s]), GD.bf16(d["stale_Cr"][s])
        y = O.native_step(npool, slots, inp["xs"][s], inp["dts"][s], Br, Cr, d["A"], d["D"], d["dt_bias"], 1e-3)
        assert torch.equal(y, d["stale_y"][s]), f"step {s}"
    assert torch.equal(npool.state[:, [0, 9]], d["stale_state_final_h0_h9"])
    assert int(npool.t[0]) == int(d["stale_t_final"])


def test_rotation_of_golden_inputs():
    for mode in ("stale", "corr", "coldoff"):
        d, inp, b, H, P, N, G, pb, c = _native_run(mode)
        for s in range(inp["steps"]):
            Br = O.rot_flat(inp["Bs"][s].reshape(b, G * N), d["R"], "fp32").reshape(b, G, N)
            Cr = O.rot_flat(inp["Cs"][s].reshape(b, G * N), d["R"], "fp32").reshape(b, G, N)
            assert torch.equal(Br.view(torch.int16), d[f"{mode}_Br"][s])
            assert torch.equal(Cr.view(torch.int16), d[f"{mode}_Cr"][s])


def test_replay_semantics_vs_v4_decode_all_modes():
    for mode in ("stale", "corr", "coldoff"):
        d, inp, b, H, P, N, G, pb, c = _native_run(mode)
        pool = O.TieredPoolRef(b, H, P, N, G, pb, c, torch.float32, torch.bfloat16)
        slots = torch.arange(b)
        O.prefill_split(pool, slots, inp["s0"])
        for s in range(inp["steps"]):
            Br, Cr = GD.bf16(d[f"{mode}_Br"][s]), GD.bf16(d[f"{mode}_Cr"][s])
            y = O.tiered_step(pool, slots, inp["xs"][s], inp["dts"][s], Br, Cr, d["A"], d["D"],
                              d["dt_bias"], 1e-3, mode=mode)
            torch.testing.assert_close(y, d[f"{mode}_y"][s], rtol=0, atol=REPLAY_ATOL, msg=lambda m: f"{mode} step {s}: {m}")
            if mode == "coldoff" or (mode == "stale" and s < c):   # no replay involved yet: exact
                assert torch.equal(y, d[f"{mode}_y"][s]), f"{mode} step {s} not exact"
        if mode == "stale":
            st = O.materialize(pool, slots, d["A"])[:, [0, 9]]
            torch.testing.assert_close(st, d["stale_state_final_h0_h9"], rtol=0, atol=REPLAY_ATOL)


def test_vllm_fp8_prefill_and_readout_bitexact():
    d = GD.load("vllm_fp8.npz")
    inp = GD.vllm_inputs()
    GD.check_sums(d, inp)
    cfg = inp["cfg"]
    S, H, P, N, G, pb, c = (cfg[k] for k in ("S", "H", "P", "N", "G", "pb", "c"))
    slots = inp["slots"]
    pool = O.TieredPoolRef(S, H, P, N, G, pb, c, O.FP8, torch.bfloat16)
    npool = O.NativePoolRef(S, H, P, N, pb, c, O.FP8)
    O.prefill_split(pool, slots, inp["s0"])
    O.prefill_split(npool, slots, inp["s0"])
    assert torch.equal(pool.cold[slots].view(torch.uint8), d["pre_codes"])
    assert torch.equal(pool.scale[slots], d["pre_scale"])
    fi = 0
    for s in range(inp["steps"]):
        args = (inp["xs"][s], inp["dts"][s], inp["Bs"][s], inp["Cs"][s], d["A"], d["D"], d["dt_bias"], None)
        yn = O.native_step(npool, slots, *args)
        yt = O.tiered_step(pool, slots, *args)
        assert torch.equal(yn, d["y"][s]), f"native step {s}"
        assert torch.equal(npool.t[slots], d["t"][s]) and torch.equal(npool.glog[slots], d["glog"][s])
        assert torch.equal(pool.t[slots], d["t"][s]) and torch.equal(pool.glog[slots], d["glog"][s])
        if s < c:                                  # replay == native until the first flush
            assert torch.equal(yt, d["y"][s]), f"replay step {s}"
        if (s + 1) % c == 0:
            assert torch.equal(npool.snap[slots].view(torch.uint8), d["flush_codes"][fi])
            assert torch.equal(npool.scale[slots], d["flush_scale"][fi])
            fi += 1
    assert fi == d["flush_codes"].shape[0]


def test_conv_step_and_state_op_vs_v4_decode():
    d = GD.load("native_decode_conv.npz")
    cfg, inp = GD.conv_case()
    for k in ("xbc", "dts", "state", "weight", "bias", "s0"):
        assert float(d[f"sum_{k}"]) == GD.MG.checksum(inp[k]), k
    b, H, P, N, G, pb, c = (cfg[k] for k in ("b", "H", "P", "N", "G", "pb", "c"))
    I = H * P
    pool = O.TieredPoolRef(b, H, P, N, G, pb, c, torch.float32, torch.float32)
    slots = torch.arange(b)
    O.prefill_split(pool, slots, inp["s0"])
    conv_state = inp["state"].clone()
    worst = 0.0
    for s in range(cfg["steps"]):
        out = O.conv_step(conv_state, slots, inp["xbc"][s], inp["weight"], inp["bias"], "silu")
        x, Bv, Cv = O.conv_split(out, I, G, N, d["R"], torch.float32)
        y = O.tiered_step(pool, slots, x.reshape(b, H, P), inp["dts"][s], Bv, Cv, d["A"], d["D"],
                          d["dt_bias"], 1e-3)
        worst = max(worst, float((y - d["y"][s]).abs().max()))
        torch.testing.assert_close(y, d["y"][s], rtol=1e-5, atol=1e-5, msg=lambda m: f"step {s}: {m}")
    assert torch.equal(conv_state, d["conv_state_final"])
    st = O.materialize(pool, slots, d["A"])[:, [0, 9]]
    torch.testing.assert_close(st, d["state_final_h0_h9"], rtol=1e-5, atol=1e-5)
