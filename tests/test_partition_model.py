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
