"""The streamed kernels' index arithmetic, restated in Python and checked on many shapes (no GPU).

The grid rule (select_internal.h: stream_ctas), the ranges (select_stream.cuh: split_point, range_of),
the row segments (make_segment), the split-row record slots and tickets (record_slot), and the CTC
grid and tickets (select_ctc.cu) decide which CTA reads which bytes and where partial results meet.
These tests restate those formulas and check their invariants on a grid of shapes: the ranges
partition the element space, every row's pieces are consecutive CTAs that cover the row exactly once,
record slots and tickets never collide, and whole-row grids give every CTA the same number of rows.
compute-sanitizer is not available on this pool; these checks stand in for it on the indexing.
"""
import itertools

import pytest

SPLIT_ALIGN = 64          # kStreamSplitAlign
MIN_RANGE = 8192          # kStreamMinRange
MAX_CTAS = 1024           # kStreamMaxCtas
TICKET_SLOTS = 2 * MAX_CTAS
CTC_MAX_UTT_PER_CTA = 64  # kMaxUttPerCta


def stream_ctas(rows, width, slots):
    g = min(slots, MAX_CTAS)
    g = min(g, rows * width // MIN_RANGE)
    g = max(g, 1)
    if rows >= g:
        per = -(-rows // g)
        g = -(-rows // per)
    return g


def split_point(rows, width, ctas, c):
    total = rows * width
    if c >= ctas:
        return total
    if rows >= ctas:
        return (c * rows // ctas) * width
    p = c * total // ctas
    return p - p % SPLIT_ALIGN


def range_of(rows, width, ctas, e):
    total = rows * width
    c = min(e * ctas // total, ctas - 1)
    while c + 1 < ctas and split_point(rows, width, ctas, c + 1) <= e:
        c += 1
    while c > 0 and split_point(rows, width, ctas, c) > e:
        c -= 1
    return c


def segment(rows, width, ctas, c, row):
    lo, hi = split_point(rows, width, ctas, c), split_point(rows, width, ctas, c + 1)
    rs = row * width
    j0 = max(lo, rs) - rs
    j1 = min(hi, rs + width) - rs
    if rs >= lo and rs + width <= hi:
        return j0, j1, 0, 1, c
    c0 = range_of(rows, width, ctas, rs)
    c1 = range_of(rows, width, ctas, rs + width - 1)
    return j0, j1, c - c0, c1 - c0 + 1, c0


def record_slot(rows, width, ctas, c, row):
    return 2 * c + (0 if row == split_point(rows, width, ctas, c) // width else 1)


ROWS = [1, 2, 3, 7, 16, 100, 127, 128, 147, 148, 149, 295, 296, 297, 1000, 1024, 4096]
WIDTHS = [1, 63, 64, 1000, 8191, 8192, 8193, 32768, 70001, 151936, 262144]
SLOTS = [148, 296]  # one CTA per SM (the warp-specialised sampler), two per SM (argmax, the wide sampler)


@pytest.mark.parametrize("slots", SLOTS)
def test_ranges_segments_records_and_tickets(slots):
    checked = 0
    for rows, width in itertools.product(ROWS, WIDTHS):
        ctas = stream_ctas(rows, width, slots)
        assert 1 <= ctas <= min(slots, MAX_CTAS)
        total = rows * width
        pts = [split_point(rows, width, ctas, c) for c in range(ctas + 1)]
        assert pts[0] == 0 and pts[-1] == total
        assert all(a < b for a, b in zip(pts, pts[1:])), (rows, width, "an empty range")
        if rows >= ctas:
            # whole rows: every CTA holds ceil(rows / ctas) or one row fewer, and no row is split
            counts = [(pts[c + 1] - pts[c]) // width for c in range(ctas)]
            assert all(p % width == 0 for p in pts)
            assert max(counts) == -(-rows // ctas) and min(counts) >= max(counts) - 1
        covered = {}  # row -> list of (j0, j1, index, count, first_cta, c)
        slots_used = set()
        tickets = {}
        for c in range(ctas):
            lo, hi = pts[c], pts[c + 1]
            r0, r1 = lo // width, (hi - 1) // width
            for r in range(r0, r1 + 1):
                j0, j1, idx, cnt, first = segment(rows, width, ctas, c, r)
                assert 0 <= j0 < j1 <= width
                covered.setdefault(r, []).append((j0, j1, idx, cnt, first, c))
                if cnt > 1:
                    slot = record_slot(rows, width, ctas, c, r)
                    assert slot < 2 * MAX_CTAS and slot not in slots_used
                    slots_used.add(slot)
                    t = record_slot(rows, width, ctas, first, r)
                    assert tickets.setdefault(t, r) == r, "two split rows share a ticket"
        assert sorted(covered) == list(range(rows))
        for r, segs in covered.items():
            segs.sort(key=lambda s: s[0])
            assert segs[0][0] == 0 and segs[-1][1] == width
            assert all(a[1] == b[0] for a, b in zip(segs, segs[1:])), "gap or overlap inside a row"
            cnt, first = segs[0][3], segs[0][4]
            assert all(s[3] == cnt and s[4] == first for s in segs) and len(segs) == cnt
            assert [s[5] for s in segs] == list(range(first, first + cnt))
            assert [s[2] for s in segs] == list(range(cnt))
        checked += 1
    assert checked == len(ROWS) * len(WIDTHS)


def ctc_grid(n_utt, n_frames, sms):
    grid = sms * 4
    grid = max(grid, -(-n_utt // (CTC_MAX_UTT_PER_CTA - 2)))
    grid = min(grid, TICKET_SLOTS, n_utt * n_frames)
    return grid


@pytest.mark.parametrize("n_utt,n_frames", list(itertools.product([1, 2, 5, 32, 100, 600, 4000],
                                                                  [1, 3, 17, 100, 1500, 3000])))
def test_ctc_ranges_and_tickets(n_utt, n_frames):
    G = ctc_grid(n_utt, n_frames, 148)
    total = n_utt * n_frames
    start = [c * total // G for c in range(G + 1)]
    assert start[0] == 0 and start[-1] == total
    split_first = {}  # CTA holding an utterance's first frame -> that (split) utterance
    whole = [0] * G
    for u in range(n_utt):
        a, b = u * n_frames, (u + 1) * n_frames
        holders = [c for c in range(G) if start[c] < b and start[c + 1] > a]
        assert holders == list(range(holders[0], holders[-1] + 1))
        if len(holders) == 1:
            whole[holders[0]] += 1
        else:
            first = holders[0]
            assert start[first] <= a < start[first + 1]
            assert first not in split_first, "two split utterances start in one CTA: ticket clash"
            split_first[first] = u
    # a CTA collapses its whole utterances plus at most one split utterance it completes
    assert max(whole) <= CTC_MAX_UTT_PER_CTA - 2


RING_FRAMES = 8           # select_ctc.cu: kRingFrames
RING_MAX_STAGE = 36864    # kRingMaxStageBytes
MAX_UTT_PER_CTA = 64      # kMaxUttPerCta


def ring_eligible(n_utt, n_frames, n_classes, esz, sms=148):
    G = 2 * sms
    total = n_utt * n_frames
    t8 = total - total % RING_FRAMES
    max_range = (t8 + G - 1) // G + 2 * RING_FRAMES
    return RING_FRAMES * n_classes * esz <= RING_MAX_STAGE and G <= TICKET_SLOTS and \
        max_range <= (MAX_UTT_PER_CTA - 2) * n_frames


def ring_start(c, t8, G, total):
    if c >= G:
        return total
    p = c * t8 // G
    return p - p % RING_FRAMES


@pytest.mark.parametrize("n_utt,n_frames", list(itertools.product([1, 2, 5, 32, 100, 600, 4000],
                                                                  [1, 3, 7, 8, 17, 100, 1500, 3000])))
@pytest.mark.parametrize("n_classes,esz", [(1025, 4), (1025, 2), (51865 // 16, 4), (1, 4), (3, 2)])
def test_ctc_ring_ranges_and_tickets(n_utt, n_frames, n_classes, esz):
    """The ring CTC kernel (select_ctc.cu: ctc_ring_kernel, launch_ctc): every stage is one bulk copy of
    eight whole frames starting on a 16-byte boundary, the ranges cover every frame once, and the
    split-utterance tickets and the per-CTA collapse list stay within their bounds."""
    if not ring_eligible(n_utt, n_frames, n_classes, esz):
        return
    G, total = 2 * 148, n_utt * n_frames
    t8 = total - total % RING_FRAMES
    row = n_classes * esz
    assert (RING_FRAMES * row) % 16 == 0                    # each stage: a legal bulk-copy size
    lo = [ring_start(c, t8, G, total) for c in range(G)]
    ring_hi = [ring_start(c + 1, t8, G, total) if c + 1 < G else t8 for c in range(G)]
    hi = [ring_hi[c] if c + 1 < G else total for c in range(G)]
    assert lo[0] == 0 and hi[-1] == total
    assert all(hi[c] == lo[c + 1] for c in range(G - 1))    # contiguous, no gap, no overlap
    for c in range(G):
        assert lo[c] <= ring_hi[c] <= hi[c]
        assert lo[c] % RING_FRAMES == 0 and (ring_hi[c] - lo[c]) % RING_FRAMES == 0
        assert (lo[c] * row) % 16 == 0                      # stage sources 16-byte aligned
        assert hi[c] - ring_hi[c] < RING_FRAMES and (c == G - 1 or hi[c] == ring_hi[c])
    split_first = {}
    whole = [0] * G
    for u in range(n_utt):
        a, b = u * n_frames, (u + 1) * n_frames
        holders = [c for c in range(G) if lo[c] < b and hi[c] > a]
        assert holders == list(range(holders[0], holders[-1] + 1))
        if len(holders) == 1:
            whole[holders[0]] += 1
        else:
            first = holders[0]
            assert first not in split_first, "two split utterances start in one CTA: ticket clash"
            split_first[first] = u
            assert first < TICKET_SLOTS
    # a CTA collapses its whole utterances and at most the two split ones it touches (first, last):
    # CtcShared.last_utt holds kMaxUttPerCta
    assert max(whole) + 2 <= MAX_UTT_PER_CTA
