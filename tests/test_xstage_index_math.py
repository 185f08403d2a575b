"""Index arithmetic of the staged-x reads in the single-column kernel
(make_planes_smem / make_q81_smem in qgemv_roofline_b200/csrc/gemv_tma.cu),
restated on the CPU.

Lane l owns the 128-byte x block at l * 128 (plus the warp's slice offset) and
reads its eight 16-byte chunks in the order (i + l) & 7; the plane words come
out in that order and three conditional shifts (by 1, 2, 4 when bit k of the
lane is set) rotate them back.  Checked here: every lane ends with chunk c in
position c, and each 16-byte read of a quarter-warp touches 8 different
4-bank groups (no shared-memory bank conflict), also for the second column of a
two-column launch, staged K * 4 bytes after the first."""

import pytest


def rotate_back(slots, lane):
    """The kernel's three conditional shifts: t[c] = pl[(c - k) & 7] if lane & k."""
    pl = list(slots)
    for k in (1, 2, 4):
        if lane & k:
            pl = [pl[(c - k) & 7] for c in range(8)]
    return pl


@pytest.mark.parametrize("lane", range(32))
def test_rotation_restores_chunk_order(lane):
    read_order = [(i + lane) & 7 for i in range(8)]  # chunk held in slot i
    assert sorted(read_order) == list(range(8))
    assert rotate_back(read_order, lane) == list(range(8))


# slice offsets of the first column, and of the second column of a two-column
# launch (staged at byte K * 4: K = 4096 and K = 11008, K % 256 == 0)
@pytest.mark.parametrize("slice_base", [0, 4096, 8192, 16384 + 4096, 44032, 44032 + 8192])
def test_quarter_warp_reads_are_conflict_free(slice_base):
    for i in range(8):
        for q in range(4):  # quarter-warps: a 16-byte access per lane, 8 lanes per wavefront
            groups = set()
            for lane in range(8 * q, 8 * q + 8):
                addr = slice_base + lane * 128 + (((i + lane) & 7) << 4)
                groups.add((addr // 16) % 8)  # 16 bytes = 4 banks; 8 groups of 4 banks
            assert len(groups) == 8
