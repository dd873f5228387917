"""Model of the GPU work partition (csrc/pp_engine.cuh) on the CPU.

Checks the index arithmetic of the split-K reduction: every unit of every
tile reaches exactly one final store, partial slots never collide, at most
two tiles per CTA go through the workspace, and the counter index (the
tile's last contributing CTA) is unique per shared tile.  CPU only.
"""
import pytest

def rs(U, parts, i): return (U * i) // parts
def pou(x, U, G):
    c = ((x + 1) * G + U - 1) // U - 1
    return min(c, G - 1)
def simulate(U, upt, G, NW):
    tiles = U // upt
    assert tiles * upt == U
    stores = {}
    slots = {}          # (cta, which) -> {tile: set(units)}
    for b in range(G):
        cu0, cu1 = rs(U, G, b), rs(U, G, b + 1)
        if cu0 >= cu1: continue
        R = cu1 - cu0
        red = {}
        for w in range(NW):
            wu0, wu1 = cu0 + rs(R, NW, w), cu0 + rs(R, NW, w + 1)
            if wu0 >= wu1: continue
            t = wu0 // upt; kc = wu0 - t * upt; t_first = t
            acc = set()
            u = wu0
            while True:
                acc.add(u)
                nt, nkc = t, kc + 1
                if nkc == upt: nkc, nt = 0, t + 1
                tile_end = nkc == 0; last = u + 1 == wu1
                if tile_end or last:
                    whole = t * upt >= wu0 and tile_end
                    if whole:
                        assert t not in stores; stores[t] = acc
                    else:
                        which = 0 if t == t_first else 1
                        assert (w, which) not in red
                        red[(w, which)] = (t, acc)
                    acc = set()
                t, kc = nt, nkc
                u += 1
                if u >= wu1: break
        ct0, ct1 = cu0 // upt, (cu1 - 1) // upt
        pend = []
        for tt in range(ct0, ct1 + 1):
            a, bb = tt * upt, tt * upt + upt
            wf = pou(max(a, cu0) - cu0, R, NW); wl = pou(min(bb, cu1) - 1 - cu0, R, NW)
            one = wf == wl and a >= cu0 + rs(R, NW, wf) and bb <= cu0 + rs(R, NW, wf + 1)
            whole = a >= cu0 and bb <= cu1
            if one and whole: continue
            s = set()
            for w in range(wf, wl + 1):
                ws0 = cu0 + rs(R, NW, w)
                if ws0 == cu0 + rs(R, NW, w + 1): continue
                which = 0 if ws0 >= a else 1
                t_, acc = red[(w, which)]
                assert t_ == tt, (t_, tt)
                assert not (s & acc); s |= acc
            if whole:
                assert tt not in stores; stores[tt] = s
            else:
                key = (b, 0 if tt == ct0 else 1)
                assert key not in slots; slots[key] = (tt, s)
                pend.append(tt)
        assert len(pend) <= 2
    # cross-CTA
    done = set()
    for key, (tt, s) in slots.items():
        if tt in done: continue
        cf, cl = pou(tt * upt, U, G), pou(tt * upt + upt - 1, U, G)
        tot = set()
        for c in range(cf, cl + 1):
            w = 1 if (c == cf and rs(U, G, c) < tt * upt) else 0
            t_, s2 = slots[(c, w)]
            assert t_ == tt
            assert not (tot & s2); tot |= s2
        assert tt not in stores; stores[tt] = tot; done.add(tt)
    for t in range(tiles):
        assert stores[t] == set(range(t * upt, t * upt + upt)), t
    # counters: c_last unique per shared tile
    cl_used = [pou(t * upt + upt - 1, U, G) for t in range(tiles) if pou(t*upt, U, G) != pou(t*upt+upt-1, U, G)]
    assert len(cl_used) == len(set(cl_used))


@pytest.mark.parametrize("upt", [1, 2, 3, 5, 16, 32, 33, 172])
@pytest.mark.parametrize("NW", [5, 6, 8, 10, 12, 16])
def test_partition_covers_every_unit_once(upt, NW):
    for tiles in [1, 2, 3, 7, 32, 64, 257]:
        U = upt * tiles
        want = max(1, -(-U // (2 * NW)))
        for G in sorted({1, 2, 3, min(148, want), min(148, U)}):
            if G <= U:
                simulate(U, upt, G, NW)


# ---------------------------------------------------------------- TMA engine
# Model of the TMA engine's warp-level protocol (csrc/pp_engine.cuh:
# UnitSeq, close_split, cta_tables_init): unit order per warp, split-tile
# arrival counters by first toucher, sums in warp order, the cross-CTA
# workspace protocol.
class UnitSeq:
    def __init__(self, wu0, wu1, upt):
        tf, tl = wu0 // upt, (wu1 - 1) // upt
        hf = (tf + 1) * upt
        head_whole = wu0 == tf * upt and wu1 >= hf
        split_tail = tl > tf and wu1 < (tl + 1) * upt
        a0, b0 = (tl * upt if split_tail else wu1), wu1
        a1, b1 = wu0, (wu0 if head_whole else min(wu1, hf))
        a2, b2 = b1, (tl * upt if split_tail else wu1)
        self.segs = [(a0, b0), (a1, b1), (a2, b2)]
        self.upt = upt

    def units(self):
        for seg, (a, b) in enumerate(self.segs):
            for u in range(a, b):
                yield seg, u, u + 1 == b


def plan_cta_starts(tiles, upt, G, slack):
    """pp_engine.cuh plan_cta_starts: whole tiles on min(G, tiles) CTAs when
    its busiest CTA holds at most `slack` units more than the equal split's
    busiest, else the equal split over G.  Returns (starts, aligned, grid)."""
    U = tiles * upt
    split_max = -(-U // G)
    G2 = min(G, tiles)
    if -(-tiles // G2) * upt <= split_max + slack:
        return [tiles * c // G2 * upt for c in range(G2 + 1)], True, G2
    return [U * c // G for c in range(G + 1)], False, G


def cta_of_unit(starts, G, x):
    """Largest c < G with starts[c] <= x (binary search in the kernel)."""
    lo, hi = 0, G - 1
    while lo < hi:
        mid = (lo + hi + 1) // 2
        if starts[mid] <= x:
            lo = mid
        else:
            hi = mid - 1
    return lo


def simulate_tma(U, upt, G, NW, starts=None):
    tiles = U // upt
    if starts is None:
        starts = [rs(U, G, b) for b in range(G + 1)]
    stores, gslots, counters = {}, {}, {}
    for b in range(G):
        cu0, cu1 = starts[b], starts[b + 1]
        assert cu0 < cu1
        R = cu1 - cu0
        wstart = [cu0 + rs(R, NW, i) for i in range(NW + 1)]
        wtile = [x // upt for x in wstart]
        red, arrivals, closers = {}, {}, {}
        for w in range(NW):
            wu0, wu1 = wstart[w], wstart[w + 1]
            if wu0 >= wu1:
                continue
            seen, acc = [], set()
            for seg, u, seg_end in UnitSeq(wu0, wu1, upt).units():
                seen.append(u)
                acc.add(u)
                t, kc = u // upt, u % upt
                if seg == 2:
                    if kc + 1 == upt:
                        assert acc == set(range(t * upt, t * upt + upt))
                        assert t not in stores
                        stores[t] = acc
                        acc = set()
                elif seg_end:
                    which = 1 if seg == 0 else 0
                    assert (w, which) not in red
                    red[(w, which)] = (t, acc)
                    acc = set()
                    x0, x1 = max(t * upt, cu0), min(t * upt + upt, cu1)
                    wf = w
                    while wf > 0 and wstart[wf] > x0:
                        wf -= 1
                    n, ww = 0, wf
                    while ww < NW and wstart[ww] < x1:
                        n += wstart[ww + 1] > wstart[ww]
                        ww += 1
                    idx = 2 * wf + (0 if wtile[wf] == t else 1)
                    arrivals.setdefault(idx, []).append((t, n, wf, x1))
            assert sorted(seen) == list(range(wu0, wu1))
            assert acc == set()
        # close every split tile (whoever is last sums the same slots)
        for idx, arr in arrivals.items():
            t, n, wf, x1 = arr[0]
            assert all(a == arr[0] for a in arr), arr
            assert len(arr) == n, (arr, n)
            s, ww = set(), wf
            while ww < NW and wstart[ww] < x1:
                if wstart[ww + 1] > wstart[ww]:
                    t_, part = red[(ww, 0 if wtile[ww] == t else 1)]
                    assert t_ == t and not (s & part)
                    s |= part
                ww += 1
            assert s == set(range(max(t * upt, cu0), min(t * upt + upt, cu1)))
            if t * upt >= cu0 and t * upt + upt <= cu1:
                assert t not in stores
                stores[t] = s
            else:
                key = (b, 0 if t == wtile[0] else 1)
                assert key not in gslots
                gslots[key] = (t, s)
                cf, cl = cta_of_unit(starts, G, t * upt), cta_of_unit(starts, G, t * upt + upt - 1)
                counters.setdefault(cl, []).append((t, cf))
    for cl, arr in counters.items():
        t, cf = arr[0]
        assert all(a == arr[0] for a in arr) and len(arr) == cl - cf + 1
        tot = set()
        for c in range(cf, cl + 1):
            t_, s = gslots[(c, 1 if (c == cf and starts[c] < t * upt) else 0)]
            assert t_ == t and not (tot & s)
            tot |= s
        assert t not in stores
        stores[t] = tot
    for t in range(tiles):
        assert stores[t] == set(range(t * upt, t * upt + upt)), t


@pytest.mark.parametrize("upt", [1, 2, 3, 5, 16, 32, 33, 172])
@pytest.mark.parametrize("NW", [4, 8, 12, 16])
def test_tma_engine_closes_every_tile_once(upt, NW):
    for tiles in [1, 2, 3, 7, 32, 64, 257]:
        U = upt * tiles
        want = max(1, -(-U // (2 * NW)))
        for G in sorted({1, 2, 3, min(148, want), min(148, U)}):
            if G <= U:  # the host never plans more CTAs than units
                simulate_tma(U, upt, G, NW)


@pytest.mark.parametrize("upt", [1, 3, 16, 32, 172])
@pytest.mark.parametrize("NW", [4, 8, 12, 16])
def test_tma_engine_with_host_cta_table(upt, NW):
    """The host's CTA-start table, in both modes, as quad_plan builds it."""
    for tiles in [1, 5, 32, 256, 1376]:
        U = upt * tiles
        G = min(148, max(1, -(-U // (2 * NW))))
        st, aligned, G = plan_cta_starts(tiles, upt, G, 32)
        assert all(st[c] < st[c + 1] for c in range(G))    # no empty CTA
        if aligned:
            assert all(x % upt == 0 for x in st)
        simulate_tma(U, upt, G, NW, starts=st)
        if aligned:
            pass  # no tile crossed a CTA boundary: simulate_tma stored every tile in-CTA


def test_sweep_shapes_plan():
    """Which BASELINE shapes get tile-aligned CTA ranges (16 warps, 148 SMs)."""
    plans = {}
    for (K, N) in [(2048, 2048), (2048, 11008), (11008, 2048), (2048, 256)]:
        tiles, upt = -(-N // 8), -(-K // 64)
        U = tiles * upt
        G = min(148, -(-U // 32))
        _, al, G = plan_cta_starts(tiles, upt, G, 32)
        plans[(K, N)] = (G, al)
    assert plans[(2048, 256)] == (32, True)
    assert plans[(2048, 2048)] == (148, True)
    assert plans[(2048, 11008)] == (148, True)
    assert plans[(11008, 2048)] == (148, False)


def test_narrow_tall_keeps_every_sm():
    """Fewer tiles than SMs must not shrink the grid when tiles are long: the
    dual kernel's 11008 x 2048 (32 tiles of 688 units) keeps 148 CTAs."""
    tiles, upt = 2048 // 64, 11008 // 16
    G = min(148, -(-tiles * upt // 32))
    st, aligned, G2 = plan_cta_starts(tiles, upt, G, 32)
    assert (G2, aligned) == (148, False)
    assert max(b - a for a, b in zip(st, st[1:])) <= -(-tiles * upt // 148)
    # short tiles with few of them: whole tiles win
    st, aligned, G2 = plan_cta_starts(32, 32, 32, 32)
    assert (G2, aligned) == (32, True)
