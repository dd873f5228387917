"""Model of the plug window slots of the tcgen05 batched kernel (``quad_tc.cu``).

A CTA multiplies stages c0 .. c0 + nst - 1 of 16 columns; four stages form a
64-column window whose plug segments the producer copies into one of two
window slots (slot = (window - first window) mod 2).  The producer issues a
window's copies together with the code copy of its first stage; for a stage
r >= S (S code slots) it first waits until stage r - S has been multiplied,
which in turn needs every stage up to r - S decoded (the MMA warp takes the
stages in order and waits for each one's decoded tiles).  Decoders read a
window's slot while they decode its stages.

The model checks the property the kernel relies on without a barrier of its
own: when a slot is refilled, every stage of the window that used it before
has been decoded -- for every split start c0, stage count and S up to 5
(the kernel caps S at 4 when plugs are present), and it shows that S = 6
would break it.
"""
from __future__ import annotations


def _windows(c0: int, nst: int):
    """(stage r at which the producer issues it, window) for the CTA's windows."""
    out = []
    for r in range(nst):
        if r == 0 or (c0 + r) % 4 == 0:
            out.append((r, (c0 + r) // 4))
    return out


def _last_stage(c0: int, nst: int, w: int) -> int:
    return max(r for r in range(nst) if (c0 + r) // 4 == w)


def _reuse_safe(c0: int, nst: int, S: int) -> bool:
    wins = _windows(c0, nst)
    w0 = wins[0][1]
    for r, w in wins:
        prev = w - 2               # the window that used the same slot before
        if prev < w0:
            continue               # first use of the slot
        if r < S:
            return False           # a prologue issue cannot wait for anything
        done_upto = r - S          # stages decoded when the producer may issue
        if _last_stage(c0, nst, prev) > done_upto:
            return False
    return True


def test_slot_reuse_needs_no_barrier_up_to_five_code_slots():
    for S in range(1, 6):
        for c0 in range(8):
            for nst in range(1, 48):
                assert _reuse_safe(c0, nst, S), (S, c0, nst)


def test_six_code_slots_would_race():
    assert any(not _reuse_safe(c0, nst, 6) for c0 in range(8) for nst in range(1, 48))


def test_prologue_issues_at_most_two_windows():
    # stages 0 .. S-1 go out before any wait: their windows must use distinct slots
    for S in range(1, 5):
        for c0 in range(8):
            for nst in range(1, 48):
                first = [w for r, w in _windows(c0, nst) if r < S]
                assert len(first) <= 2 and len(set(w % 2 for w in first)) == len(first), (S, c0, nst)
