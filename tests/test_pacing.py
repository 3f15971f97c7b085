"""Device-paced link emulation (``nvlink`` bandwidth mode): cost model, harness wiring, the calls the
NVLink collectives and the ZeRO-3 gathers make (CPU), and the paced hold on one GPU."""

from __future__ import annotations

import pytest
import torch

from cs244c_llama_zero_b200.experiments import harness
from cs244c_llama_zero_b200.parallel.comm import pacing


def test_cost_model_and_env():
    assert pacing.pacing_from_env({}) is None
    assert pacing.pacing_from_env({pacing.ENV_BW: "0"}) is None
    assert pacing.pacing_from_env({pacing.ENV_BW: "10"}) == (10.0, 0.0)
    assert pacing.pacing_from_env({pacing.ENV_LATENCY: "0.5"}) == (0.0, 0.5)
    # ring volumes per GPU link
    assert pacing.link_bytes("allreduce", 1000, 4) == 1500
    assert pacing.link_bytes("reduce_scatter", 1000, 4) == 750
    assert pacing.link_bytes("allgather", 1000, 4) == 750
    assert pacing.link_bytes("allreduce", 1000, 1) == 0
    # 1 Gbit/s: 125 MB/s -> 1 MB takes 8 ms; latency adds on top
    assert pacing.pace_cost_ns(1_000_000, 1.0, 0.0) == 8_000_000
    assert pacing.pace_cost_ns(1_000_000, 1.0, 2.0) == 10_000_000
    assert pacing.pace_cost_ns(123, 0.0, 0.0) == 0


def test_native_cost_matches_python_model():
    from cs244c_llama_zero_b200 import ops

    ext = ops.load_extension()
    for nbytes, gbps, lat in ((1 << 20, 1.0, 0.0), (12_345_678, 25.0, 0.25), (0, 0.0, 1.0), (999, 3.3, 0.0)):
        assert ext.pace_cost_ns(nbytes, gbps, lat) == pacing.pace_cost_ns(nbytes, gbps, lat)


def test_harness_nvlink_mode_env_and_validation(tmp_path):
    args = harness.parse_args(["--results-dir", str(tmp_path), "--name", "t", "--bandwidth-mode", "nvlink",
                               "--bandwidth-gbps", "5", "--sim-latency-ms", "0.1", "--collective-impl", "nvls"])
    case = harness._build_cases(args)[0]
    env = harness._build_launch_env(case)
    assert env[pacing.ENV_BW] == "5.0" and env[pacing.ENV_LATENCY] == "0.1"
    assert "ZERO_SIM_BW_GBPS" not in env and "ZERO_SOCKET_SHAPER_BW_GBPS" not in env
    case.bandwidth_gbps = 0.0
    case.sim_latency_ms = 0.0
    env = harness._build_launch_env(case)
    assert pacing.ENV_BW not in env and pacing.ENV_LATENCY not in env
    bad = harness.parse_args(["--results-dir", str(tmp_path), "--name", "t", "--bandwidth-mode", "nvlink",
                              "--collective-impl", "torch"])
    with pytest.raises(ValueError, match="nvls or p2p"):
        harness.run_matrix(bad)


class _FakePacer:
    def __init__(self, log):
        self.log = log
        self.n = 0

    def begin(self):
        self.n += 1
        self.log.append(("begin", self.n))
        return self.n

    def end(self, slot, nbytes):
        self.log.append(("end", slot, nbytes))


class _FakeCtx:
    def __init__(self, log):
        self.log = log

    def __getattr__(self, name):
        return lambda *a: self.log.append(("kernel", name))


class _FakeBuf:
    def __init__(self, log, dtype):
        self.ctx = _FakeCtx(log)
        self.tensor = torch.zeros(1, dtype=dtype)


def test_nvlink_collectives_pace_every_transfer(monkeypatch):
    from cs244c_llama_zero_b200.parallel.comm import nvlink

    monkeypatch.setattr(nvlink, "_world", lambda: 4)
    coll = nvlink.NvlinkCollectives(device=torch.device("cpu"))
    assert coll.pacer is None  # no pacing variables in the environment
    log = []
    coll.pacer = _FakePacer(log)
    monkeypatch.setattr(coll, "_locate", lambda t: (_FakeBuf(log, t.dtype), 0))
    flat = torch.zeros(64)
    coll.allreduce_scaled_(flat, 0.25)
    coll.reduce_scatter_accumulate_(torch.zeros(16), flat, 1.0)
    coll.allgather_into(torch.zeros(64, dtype=torch.bfloat16), torch.zeros(16, dtype=torch.bfloat16))
    kinds = [e[0] for e in log]
    assert kinds == ["begin", "kernel", "end"] * 3
    ends = [e for e in log if e[0] == "end"]
    assert [e[1] for e in ends] == [1, 2, 3]
    # 64 fp32 = 256 B: all-reduce 2*3/4*256, reduce-scatter 3/4*256; all-gather of 4 x 32 B shards: 3*32
    assert [e[2] for e in ends] == [384, 192, 96]


def test_stage3_gathers_share_the_pacer():
    from cs244c_llama_zero_b200.parallel.zero.base import CommClock
    from cs244c_llama_zero_b200.parallel.zero.stage3 import _PullGather

    class Native:
        pacer = "unset"

        def set_pacer(self, p):
            self.pacer = p

    class Coll:
        pacer = object()

        def locate_symmetric(self, t):
            return "ctx", 0

    class Eng:
        device = torch.device("cpu")
        world_size = 2
        _handle_order = []
        clock = CommClock(torch.device("cpu"))
        collectives = Coll()

    native = Native()
    _PullGather(Eng(), torch.zeros(8, dtype=torch.uint8), [torch.zeros(8, dtype=torch.uint8)], native=native)
    assert native.pacer is Coll.pacer


@pytest.mark.gpu
def test_paced_hold_on_device():
    from cs244c_llama_zero_b200 import ops

    ext = ops.load_extension()
    ext.reset_device_errors()
    # 4 Gbit/s: 2.5 MB -> 5 ms on the emulated link
    pacer = ext.LinkPacer(torch.cuda.current_device(), 4.0, 0.0, int(10e9))
    cost_ms = pacer.cost_ns(2_500_000) / 1e6
    assert cost_ms == pytest.approx(5.0)
    x = torch.randn(1 << 20, device="cuda")
    for _ in range(2):  # warm-up
        s = pacer.begin()
        x.mul_(1.0)
        pacer.end(s, 0)
    torch.cuda.synchronize()

    def timed(fn):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b)

    def one():
        s = pacer.begin()
        x.mul_(1.0)  # the "transfer": far shorter than its 5 ms cost
        pacer.end(s, 2_500_000)

    t1 = timed(one)
    assert cost_ms * 0.97 <= t1 < cost_ms + 20.0

    # Two transfers on two streams queue on the same link: about twice the cost in total.
    side = torch.cuda.Stream()

    def two():
        main = torch.cuda.current_stream()
        side.wait_stream(main)
        one()
        with torch.cuda.stream(side):
            one()
        main.wait_stream(side)

    t2 = timed(two)
    assert 2 * cost_ms * 0.97 <= t2 < 2 * cost_ms + 20.0
    assert ext.read_device_errors()[0] == 0


def test_fused_step_and_routed_entry_points_pass_the_binding_arguments(monkeypatch):
    """The NVLink collectives' fused-step and routing entry points hand the native bindings their
    arguments in the bindings' order (checked here without a GPU)."""
    from cs244c_llama_zero_b200.parallel.comm import nvlink
    from cs244c_llama_zero_b200.parallel.zero.optim import AdamWConfig

    monkeypatch.setattr(nvlink, "_world", lambda: 2)
    coll = nvlink.NvlinkCollectives(device=torch.device("cpu"))
    calls = []

    class Ctx:
        def rs_adamw_allgather(self, *args):
            calls.append(args)

    class Buf:
        multicast = False

        def __init__(self, dtype):
            self.ctx = Ctx()
            self.handle = type("H", (), {"buffer_ptrs": [4096, 8192]})()

    bufs = {torch.bfloat16: Buf(torch.bfloat16), torch.float32: Buf(torch.float32)}
    monkeypatch.setattr(coll, "_locate", lambda t: (bufs[t.dtype], 32 if t.dtype == torch.float32 else 16))
    params, grads = torch.zeros(32, dtype=torch.bfloat16), torch.zeros(32)
    master, m, v = torch.zeros(16), torch.zeros(16), torch.zeros(16)
    cfg = AdamWConfig(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    sq = torch.zeros(1)
    assert coll.reduce_scatter_adamw_allgather(params, grads, master, m, v, 0.5, cfg, 7, None, sq)
    (args,) = calls
    assert args[0] is bufs[torch.float32].ctx and args[1:4] == (32, 16, 16)  # grads ctx, g_off, param_off, chunk
    assert args[4] is master and args[5] is m and args[6] is v
    assert args[7:13] == (0.5, 1e-3, 0.9, 0.95, 1e-8, 0.1) and args[13] == 7 and args[14] is None and args[15] is sq
    assert coll.shard_bases(grads) == [4096 + 32, 8192 + 32]
