"""CTC head schedule arithmetic (qppocr_b200/csrc/gemm_tc.cu: head_lo, cta_tile,
the epilogue's per-group slots, head_cta_of and argmax_combine_kernel's slot
enumeration), restated with C integer semantics and checked exhaustively on
the CPU: every partial the combine reads is written by exactly one (CTA,
epilogue group), no two writers share a slot, and each row block's partials
cover all of its column tiles exactly once, for ragged and full-size grids."""
import pytest


def c_div(a, b):  # C integer division (truncates toward zero)
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b > 0) else -q


def c_mod(a, b):
    return a - b * c_div(a, b)


def head_lo(b, T, W):
    return c_div(b * T, W)


def head_cta_of(t, T, W):
    return c_div((t + 1) * W + T - 1, T) - 1


def writes(m_tiles, n_tiles, W, ngrp):
    """(row block, slot) -> (cta, group, tiles covered), from the GEMM side."""
    T = m_tiles * n_tiles
    out = {}
    for b in range(W):
        lo, hi = head_lo(b, T, W), head_lo(b + 1, T, W)
        for g in range(ngrp):
            cur, slot, tiles = -1, 0, []
            for t in range(lo + g, hi, ngrp):  # the epilogue group's tiles
                mb = c_div(t, n_tiles)
                if mb != cur:
                    if cur >= 0:
                        assert (cur, slot) not in out
                        out[(cur, slot)] = (b, g, tiles)
                    cur, slot, tiles = mb, t - mb * n_tiles, []
                tiles.append(t)
            if cur >= 0:
                assert (cur, slot) not in out
                out[(cur, slot)] = (b, g, tiles)
    return out


def reads(m_tiles, n_tiles, W, ngrp):
    T = m_tiles * n_tiles
    out = []
    for mb in range(m_tiles):
        t0, t1 = mb * n_tiles, mb * n_tiles + n_tiles
        for b in range(head_cta_of(t0, T, W), head_cta_of(t1 - 1, T, W) + 1):
            lo = head_lo(b, T, W)
            s0, s1 = max(lo, t0), min(head_lo(b + 1, T, W), t1)
            for g in range(ngrp):
                first = s0 + c_mod(c_mod(g - (s0 - lo), ngrp) + ngrp, ngrp)
                if first < s1:
                    out.append((mb, first - t0))
    return out


@pytest.mark.parametrize("ngrp", [1, 2])
@pytest.mark.parametrize("sms", [148, 132, 8])
@pytest.mark.parametrize("rows,n_tiles", [(1, 1), (77, 4), (128, 3), (300, 1), (300, 74), (2560, 147),
                                          (10240, 74), (10240, 147), (20000, 2)])
def test_every_partial_read_is_written_once(rows, n_tiles, sms, ngrp):
    m_tiles = (rows + 127) // 128
    T = m_tiles * n_tiles
    W = min(T, sms)  # run_kernel's grid and head_workers
    w = writes(m_tiles, n_tiles, W, ngrp)
    r = reads(m_tiles, n_tiles, W, ngrp)
    assert len(r) == len(set(r))
    assert set(r) == set(w)
    for mb in range(m_tiles):
        covered = sorted(t for (m, _), (_, _, ts) in w.items() if m == mb for t in ts)
        assert covered == list(range(mb * n_tiles, (mb + 1) * n_tiles))
    assert all(0 <= s < n_tiles for _, s in r)  # slots stay inside the n_tiles x M buffer
