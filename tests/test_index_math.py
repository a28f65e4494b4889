"""Host restatements of the index arithmetic of the split-K / split-row
kernels, checked exhaustively on the CPU for many shapes (no GPU):

* gemv_t_kernel (csrc/bnbq_gemv_xtab.cu, plan_t / gemv_t_reduce_kernel): CTA
  b of G takes units [b U / G, (b + 1) U / G) (column-group-major, R row
  blocks per group) and stores one partial per column group it touches, at
  segment g - g0(b) < maxseg; the reduction finds, for group g, the CTAs
  cta_of(g R) .. cta_of((g + 1) R - 1). Every unit must be counted exactly
  once and every partial slot read must exist.
* quant_nf4_dq_kernel's grid split (launch_dq): the nested pass gets the last
  CTAs, at most 1/16 of the grid (at least 8), and the 32 CTAs that form the
  mean's slot sums are NF4-pass CTAs."""
from __future__ import annotations

import itertools

import pytest


def plan_t(n_rows: int, k: int, sm_count: int):
    rbs = (n_rows + 31) // 32
    units = (k // 256) * rbs
    grid = min(units, sm_count)
    maxseg = 1
    for b in range(grid):
        u0, u1 = b * units // grid, (b + 1) * units // grid
        maxseg = max(maxseg, (u1 - 1) // rbs - u0 // rbs + 1)
    return rbs, units, grid, maxseg


def cta_of(u: int, units: int, grid: int) -> int:
    return ((u + 1) * grid + units - 1) // units - 1


@pytest.mark.parametrize("n_rows,k,sms", list(itertools.product(
    [1, 31, 32, 33, 100, 256, 512, 777, 1000, 4096, 14336, 28672], [256, 512, 768, 4096, 14336], [148, 132, 7])))
def test_backward_partials_cover_every_unit_once(n_rows, k, sms):
    rbs, units, grid, maxseg = plan_t(n_rows, k, sms)
    groups = k // 256
    ranges = [(b * units // grid, (b + 1) * units // grid) for b in range(grid)]
    for u in range(units):  # the CTA that holds each unit
        b = cta_of(u, units, grid)
        assert ranges[b][0] <= u < ranges[b][1]
    counted = [0] * units
    for g in range(groups):
        lo, hi = cta_of(g * rbs, units, grid), cta_of((g + 1) * rbs - 1, units, grid)
        for b in range(lo, hi + 1):
            u0, u1 = ranges[b]
            seg = g - u0 // rbs
            assert 0 <= seg < maxseg
            assert seg < (u1 - 1) // rbs - u0 // rbs + 1  # a segment this CTA writes
            for u in range(max(u0, g * rbs), min(u1, (g + 1) * rbs)):
                counted[u] += 1
    assert all(c == 1 for c in counted)


def dq_split(grid_full: int, want_warps4: int, warps8: int):
    grid = max(min(grid_full, (want_warps4 + 7) // 8), 64)
    cap3 = max(grid // 16, 8)
    ctas3 = min(max((warps8 + 7) // 8, 1), cap3)
    return grid, grid - ctas3, ctas3


@pytest.mark.parametrize("n", [64, 1000, 1 << 16, 1 << 20, 4096 * 4096, 4096 * 14336, 28672 * 8192])
@pytest.mark.parametrize("per_sm", [3, 4])
def test_double_quant_grid_split(n, per_sm):
    bs, bs2 = 64, 256
    warps4 = (n + 255) // 256  # NF4 pass, blocks of <= 256: one 256-element segment per warp step
    nb = -(-n // bs)
    warps8 = (nb + 255) // 256
    grid, cta0, ctas3 = dq_split(148 * per_sm, warps4, warps8)
    if grid > 148 * per_sm:
        pytest.skip("the launch refuses this (fewer resident CTAs than the minimum grid)")
    assert cta0 >= 32  # the mean's slot CTAs run the NF4 pass
    assert 1 <= ctas3 <= max(grid // 16, 8)
    assert cta0 + ctas3 == grid
