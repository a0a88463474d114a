"""The band order of conv_pair_tc_kernel (PairStream in
rosenna_b200/csrc/conv_tc.cu), restated in Python and checked for the
properties the kernel relies on, over batches, image sizes, paddings and grid
sizes:

* every (sample tile, second-conv band) item is taken by exactly one CTA;
* a second-conv band comes after every first-conv band of its tile whose
  pooled rows it reads (its `need` count covers them);
* the first-conv band after the one `need` ends on comes before the
  second-conv band (or that one is the CTA's last first-conv band), so the
  drain, which publishes a band once the next first-conv band is stored,
  publishes it before the loader waits for it;
* no first-conv band of local tile j + 2 (which reuses local tile j's column
  of the intermediate buffer) comes before a second-conv band of tile j.

The restatement follows the device code line for line (init and next)."""
import pytest

LAG = 2

class PS:
    def __init__(s, nb2, hq1, bh2, ph2, pad2, hin2, w0, w1):
        s.nb2, s.hq1, s.bh2, s.ph2, s.pad2, s.hin2 = nb2, hq1, bh2, ph2, pad2, hin2
        s.lag = min(LAG, s.rmax(nb2 - 1) // hq1 + 1)
        if w1 <= w0:
            s.tA, s.tB, s.t1, s.t2 = 0, -1, 0, 0; return
        s.tA = w0 // nb2; s.tB = (w1 - 1) // nb2
        s.kaA = w0 - s.tA * nb2; s.kbB = w1 - s.tB * nb2
        s.t1 = s.t2 = s.tA
        s.c1 = s.c2lo = s.clo(s.tA); s.c1hi = s.chi(s.tA)
        s.pos1 = s.base1 = 0
        s.k2 = s.ka(s.tA); s.k2end = s.kb(s.tA)
    def ka(s, t): return s.kaA if t == s.tA else 0
    def kb(s, t): return s.kbB if t == s.tB else s.nb2
    def rmin(s, k): return max(k * s.bh2 - s.pad2, 0)
    def rmax(s, k): return min(k * s.bh2 - s.pad2 + s.ph2 - 1, s.hin2 - 1)
    def clo(s, t): return s.rmin(s.ka(t)) // s.hq1
    def chi(s, t): return s.rmax(s.kb(t) - 1) // s.hq1
    def next(s):
        have1 = s.t1 <= s.tB
        if s.t2 <= s.tB:
            dep = s.base1 + (s.rmax(s.k2) // s.hq1 - s.c2lo)
            if not have1 or dep + s.lag < s.pos1:
                r = (2, s.t2, s.k2, (s.t2 - s.tA) & 1, dep + 1, None, None)
                s.k2 += 1
                if s.k2 == s.k2end:
                    s.base1 += s.chi(s.t2) - s.c2lo + 1
                    s.t2 += 1
                    if s.t2 <= s.tB:
                        s.k2 = s.ka(s.t2); s.k2end = s.kb(s.t2); s.c2lo = s.clo(s.t2)
                return r
        if not have1: return None
        r = [1, s.t1, s.c1, (s.t1 - s.tA) & 1, None, s.pos1, None]
        s.pos1 += 1
        s.c1 += 1
        if s.c1 > s.c1hi:
            s.t1 += 1
            if s.t1 <= s.tB:
                s.c1 = s.clo(s.t1); s.c1hi = s.chi(s.t1)
        r[6] = s.t1 > s.tB
        return tuple(r)

def check(ntiles, Hin2, pad2, grid, bh1=4, bh2=2, ph2=4):
    Ho2 = Hin2 + 2 * pad2 - 2
    nb2 = (Ho2 + bh2 - 1) // bh2
    Hq1 = Hin2; hq1 = bh1 // 2
    nb1 = (2 * Hq1 + bh1 - 1) // bh1
    items = ntiles * nb2
    seen2 = set()
    for b in range(grid):
        w0 = items * b // grid; w1 = items * (b + 1) // grid
        ps = PS(nb2, hq1, bh2, ph2, pad2, Hin2, w0, w1)
        seq = []
        while True:
            r = ps.next()
            if r is None: break
            seq.append(r)
        done = {}  # (tile) -> set of conv1 bands computed, in order
        conv1_pos = []  # (t, band)
        for idx, r in enumerate(seq):
            if r[0] == 1:
                assert r[5] == len(conv1_pos)
                assert 0 <= r[2] < nb1
                conv1_pos.append((r[1], r[2], idx))
                # WAR: no conv2 of tile t-2 remains after this
                t = r[1]
                later2 = [q for q in seq[idx:] if q[0] == 2 and q[1] <= t - 2 and q[1] >= ps.tA]
                assert not later2, (b, r, later2[:2])
            else:
                t, k = r[1], r[2]
                assert (t, k) not in seen2
                seen2.add((t, k))
                need = r[4]
                assert need <= len(conv1_pos)
                # rows read are covered by conv1 bands of tile t computed before (same parity)
                lo = max(k * bh2 - pad2, 0); hi = min(k * bh2 - pad2 + ph2 - 1, Hin2 - 1)
                have = {bb for (tt, bb, _) in conv1_pos[:need] if tt == t}
                for row in range(lo, hi + 1):
                    assert row // hq1 in have, (b, r, row)
                # deadlock-free publishing: the drain publishes a first-conv
                # band at the end of the next first-conv band (at once for the
                # last one), which must come before this band
                dep_t, dep_b, dep_idx = conv1_pos[need - 1]
                is_last = seq[dep_idx][6]
                assert is_last or (need < len(conv1_pos) and conv1_pos[need][2] < idx), (b, r)
                # parity buffer was not overwritten by a later tile's conv1 between
                for (tt, bb, ii) in conv1_pos:
                    if ii < idx and tt != t and (tt - ps.tA) % 2 == (t - ps.tA) % 2 and tt > t:
                        raise AssertionError(("overwrite", b, r, tt))
    assert seen2 == {(t, k) for t in range(ntiles) for k in range(nb2)}, "coverage"


CASES = [(ntiles, Hin2, pad2, grid)
         for ntiles in (1, 2, 3, 5, 17, 128, 512)
         for Hin2, pad2 in ((14, 1), (14, 0), (14, 2), (7, 1), (2, 1), (3, 0), (30, 1), (1, 1))
         for grid in (1, 2, 3, 7, 148)
         if Hin2 + 2 * pad2 - 2 >= 1]


@pytest.mark.parametrize("ntiles,Hin2,pad2,grid", CASES)
def test_pair_stream_order(ntiles, Hin2, pad2, grid):
    check(ntiles, Hin2, pad2, grid)
