"""The 3xTF32 kernel's work split (wg_sgemm_tc_plan: host arithmetic, no GPU).

The persistent kernel takes whole 128 x 256 tiles for every full wave of the
grid and may cut the tiles of a partial last wave into k-segments; these tests
pin the plans of the benchmark shapes and the invariants every plan keeps.
"""
import ctypes as ct

import pytest

from wgblas_b200 import _native as nat

B200_SMS = 148


def plan(m, n, k, sms=B200_SMS):
    p = nat.TcPlan()
    nat.check(nat.lib.wg_sgemm_tc_plan(sms, m, n, k, ct.byref(p)))
    return p


def round_up(x, q):
    return (x + q - 1) // q * q


def test_headline_shape_splits_the_last_wave():
    # 4096^3: 32 x 16 = 512 tiles = 3 full waves + 68 tiles, cut in two along k.
    p = plan(4096, 4096, 4096)
    assert (p.tiles_m, p.tiles_n, p.k_blocks) == (32, 16, 256)
    assert (p.grid, p.whole_tiles, p.split_tiles, p.split_segments) == (148, 444, 68, 2)
    operands = 2 * (4096 * 4096 * 4) * 2
    assert p.workspace_bytes == operands + 68 * 2 * 128 * 256 * 4 + 68 * 4 + 256


def test_single_partial_wave_of_deep_tiles_stays_whole():
    # 2048 x 2048 x 16384 (one panel at 8 GPUs): 128 tiles on 148 SMs. Splitting
    # them measured slower on B200 than running each tile whole on its own SM.
    p = plan(2048, 2048, 16384)
    assert (p.grid, p.whole_tiles, p.split_tiles, p.split_segments) == (128, 128, 0, 1)


def test_full_waves_never_split():
    p = plan(148 * 128, 256, 4096)  # exactly one wave
    assert (p.grid, p.split_tiles) == (148, 0)
    p = plan(128 * 74, 512, 4096)  # exactly one wave again, 74 x 2 tiles
    assert (p.grid, p.split_tiles) == (148, 0)


@pytest.mark.parametrize("m,n,k", [(512, 512, 512), (1000, 1023, 777), (1, 1, 8), (4096, 4096, 4096),
                                   (16384, 2048, 16384), (8192, 8192, 8192), (300, 70000, 64),
                                   (33, 257, 100000)])
@pytest.mark.parametrize("sms", [1, 2, 132, 148, 160])
def test_plan_invariants(m, n, k, sms):
    p = plan(m, n, k, sms)
    T = p.tiles_m * p.tiles_n
    assert p.tiles_m == round_up(m, 128) // 128
    assert p.tiles_n == round_up(n, 256) // 256
    assert p.k_blocks == round_up(k, 32) // 16
    assert p.whole_tiles + p.split_tiles == T
    assert 1 <= p.grid <= sms
    if p.split_tiles:
        # only the leftover of the full waves is split, into 2..16 segments of >= 4 k-blocks
        assert p.split_tiles == T % sms
        assert 2 <= p.split_segments <= min(16, p.k_blocks // 4)
        assert p.grid <= max(p.whole_tiles, p.split_tiles * p.split_segments)
    else:
        assert p.split_segments == 1
        assert p.grid == min(T, sms)
    operands = 2 * 4 * round_up(k, 32) * (round_up(m, 128) + round_up(n, 256))
    assert p.workspace_bytes >= operands


def test_rejects_bad_arguments():
    p = nat.TcPlan()
    assert nat.lib.wg_sgemm_tc_plan(0, 64, 64, 64, ct.byref(p)) == nat.WG_ERR_INVALID_ARGUMENT
    assert nat.lib.wg_sgemm_tc_plan(148, 64, 64, 4, ct.byref(p)) == nat.WG_ERR_INVALID_ARGUMENT
    assert nat.lib.wg_sgemm_tc_plan(148, 64, 64, 64, None) == nat.WG_ERR_INVALID_ARGUMENT


def panel_plan(P, m_local, n, k, sms=B200_SMS):
    w = (ct.c_int64 * 1024)()
    cnt = ct.c_size_t()
    nat.check(nat.lib.wg_sharded_panel_plan(sms, P, m_local, n, k, w, 1024, ct.byref(cnt)))
    return [w[i] for i in range(cnt.value)]


@pytest.mark.parametrize("P", [1, 2, 4, 8])
@pytest.mark.parametrize("n,k", [(16384, 16384), (5000, 777), (300, 64), (70000, 4096)])
def test_sharded_panels_cover_n_in_tile_columns(P, n, k):
    w = panel_plan(P, max(1, 16384 // P), n, k)
    assert sum(w) == n and all(x > 0 for x in w)
    assert all(x % 256 == 0 for x in w[:-1]) and (w[-1] % 256 == 0 or w[-1] == n - sum(w[:-1]))
    assert w == panel_plan(P, max(1, 16384 // P), n, k)  # deterministic


def test_sharded_panels_at_the_benchmark_shape():
    # One rank: no broadcast to hide, so the whole product is one panel.
    assert panel_plan(1, 16384, 16384, 16384) == [16384]
    for P in (2, 4, 8):
        w = panel_plan(P, 16384 // P, 16384, 16384)
        # a short first panel (its broadcast is exposed), wider ones after it
        assert len(w) >= 2 and w[0] <= 16384 // 16 and max(w) >= 4 * w[0]


def test_sharded_panel_plan_depends_on_the_row_block():
    # Ranks with different m_local would plan differently on their own, which is
    # why a sharded call agrees on (max m_local, min SMs) before planning.
    assert panel_plan(8, 2048, 16384, 16384) != panel_plan(8, 4096, 16384, 16384)


def test_sharded_panel_plan_reports_its_length():
    w = (ct.c_int64 * 1)()
    cnt = ct.c_size_t()
    st = nat.lib.wg_sharded_panel_plan(B200_SMS, 8, 2048, 16384, 16384, w, 1, ct.byref(cnt))
    assert st == nat.WG_ERR_INVALID_ARGUMENT and cnt.value > 1
