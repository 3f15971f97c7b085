"""Host-side GEMM schedulers (no GPU needed): automatic tile choice and the grouped dgrad + wgrad plan.

The grouped plan is checked against an independent re-simulation of its boustrophedon deal and
against running the two problems as separate persistent launches.
"""

from __future__ import annotations

import math

import pytest

EPI_STORE, EPI_RESIDUAL, EPI_ROPE, EPI_SWIGLU, EPI_SWIGLU_BWD, EPI_ACC_F32 = range(6)
SMS = 148


@pytest.fixture(scope="module")
def C():
    from cs244c_llama_zero_b200 import ops

    return ops.load_extension()


SHAPES = [(8192, 768, 768), (8192, 2304, 768), (8192, 4096, 768), (8192, 768, 2048), (8192, 768, 4096),
          (4096, 768, 8192), (1280, 768, 8192), (8192, 32000, 768), (300, 136, 200), (1000, 264, 392)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_tile_choice_respects_epilogue_constraints(C, M, N, K):
    for epi in range(6):
        for b_mn in (False, True):
            bn, splits, cg = C.gemm_tile_choice(M, N, K, epi, 64, epi == EPI_ACC_F32, b_mn, SMS)
            assert bn in (128, 192, 256) and cg in (1, 2) and splits >= 1
            if epi in (EPI_ROPE, EPI_SWIGLU):
                assert bn != 192
            if epi == EPI_ROPE:
                assert (bn // 2) % 64 == 0  # whole heads per epilogue half
            if cg == 2 and b_mn:
                assert (bn // 2) % 64 == 0  # B halves of whole 64-column TMA boxes
            if epi != EPI_ACC_F32:
                assert splits == 1
            else:
                kb = math.ceil(K / 64)
                assert splits <= max(1, min(32, kb // 4))


def test_tile_choice_model_shapes(C):
    # data gradient of the MLP down projection: CTA pairs of 256 x 256 are the measured best
    assert C.gemm_tile_choice(8192, 768, 4096, EPI_STORE, 64, False, True, SMS) == [256, 1, 2]
    # fused-epilogue forwards, against the fastest variant measured on B200 (TFLOP/s in brackets):
    # the short-K residual GEMM stays on single CTAs (450 vs 410 as pairs), the others take pairs
    assert C.gemm_tile_choice(8192, 768, 768, EPI_RESIDUAL, 64, False, False, SMS) == [192, 1, 1]
    assert C.gemm_tile_choice(8192, 2048, 5504, EPI_RESIDUAL, 64, False, False, SMS) == [256, 1, 2]  # 1377
    assert C.gemm_tile_choice(8192, 4096, 768, EPI_SWIGLU, 64, False, False, SMS) == [256, 1, 2]  # 1071
    assert C.gemm_tile_choice(8192, 1280, 768, EPI_ROPE, 64, False, False, SMS) == [256, 1, 2]
    # one wave or less of units: the weight gradient splits K to fill the SMs
    bn, splits, cg = C.gemm_tile_choice(768, 768, 8192, EPI_ACC_F32, 64, True, True, SMS)
    assert splits > 1


def _simulate(units0, kbs0, units1, kbs1, pairs):
    """Boustrophedon deal of the longer units first; returns (first problem, makespan)."""
    c0, c1 = kbs0 + 3, kbs1 + 3
    first = 1 if c1 > c0 else 0
    n_first = units1 if first else units0
    costs = [c1 if first else c0] * n_first + [c0 if first else c1] * (units0 + units1 - n_first)
    load = [0] * pairs
    for u, c in enumerate(costs):
        k, r = divmod(u, pairs)
        load[pairs - 1 - r if k & 1 else r] += c
    return first, max(load)


def _separate(units, kbs, pairs):
    return math.ceil(units / pairs) * (kbs + 3)


@pytest.mark.parametrize("T,out,inp", [(8192, 4096, 768), (8192, 768, 768), (8192, 1280, 768), (8192, 32000, 768),
                                       (1000, 264, 392), (2048, 4000, 768)])
def test_grouped_plan_matches_simulation_and_beats_separate(C, T, out, inp):
    splits, kbs1, first, units_first, units_total, span, tiles0, tiles1 = C.grouped_dgrad_wgrad_plan(T, out, inp, SMS)
    pairs = SMS // 2
    kb0 = math.ceil(out / 64)  # data gradient: K = out, never split
    kb1 = math.ceil(T / 64)    # weight gradient: K = T tokens
    assert tiles0 == math.ceil(T / 256) * math.ceil(inp / 256)
    assert tiles1 == math.ceil(out / 256) * math.ceil(inp / 256)
    assert splits == math.ceil(kb1 / kbs1) and kbs1 * (splits - 1) < kb1 <= kbs1 * splits
    units1 = tiles1 * splits
    assert units_total == tiles0 + units1
    assert units_first == (units1 if first else tiles0)
    sim_first, sim_span = _simulate(tiles0, kb0, units1, kbs1, pairs)
    assert (first, span) == (sim_first, sim_span)
    # no worse than the two problems as separate launches with the same split
    assert span <= _separate(tiles0, kb0, pairs) + _separate(units1, kbs1, pairs)
    # the chosen split is the best of the candidates the planner tries
    for s in (1, 2, 3, 4, 6, 8, 12, 16):
        if s > 1 and kb1 // s < 4:
            break
        kbs = math.ceil(kb1 / s)
        assert span <= _simulate(tiles0, kb0, tiles1 * math.ceil(kb1 / kbs), kbs, pairs)[1]


def test_grouped_plan_explicit_split(C):
    splits, kbs1, *_ = C.grouped_dgrad_wgrad_plan(8192, 768, 768, SMS, 3)
    assert splits == 3 and kbs1 == math.ceil(128 / 3)
