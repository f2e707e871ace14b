"""CPU check of the grouped-GEMM work schedule (fused-moe-yws_b200/csrc/gemm_sched.cuh).

The device code is restated line for line in Python and run for every CTA of a launch over
many (tiles, K steps, grid) shapes. Checked: every tile's K range is covered exactly once;
each CTA holds at most one partial tile per partial slot (slot 0: its range starts inside
the tile, slot 1: the tile ends its range), which is what the two-slot partial buffer
assumes; the contributors of a split tile are the CTAs cta_of(first step) ..
cta_of(last step) with non-empty ranges, and their step counts add up to KS, so the
arrival counter of the first contributor reaches KS exactly once; and every CTA does its
whole tiles before its split segments.
"""
import itertools

import pytest


class StreamK:
    def __init__(self, W, G):
        self.W, self.G = W, G

    def start(self, c):
        return c * self.W // self.G

    def cta_of(self, g):
        return ((g + 1) * self.G + self.W - 1) // self.W - 1


class Schedule:
    """Schedule of gemm_sched.cuh: whole tiles first, then the stream-K split."""

    def __init__(self, num_tiles, ks, grid, c):
        self.KS, self.G, self.cta, self.num_tiles = ks, grid, c, num_tiles
        if num_tiles <= grid and 2 * num_tiles >= grid:
            self.dp_tiles = num_tiles  # G/2 .. G tiles: whole, one per CTA
        else:
            self.dp_tiles = (num_tiles // grid - 1) * grid if num_tiles > 2 * grid else 0
        self.sk = StreamK((num_tiles - self.dp_tiles) * ks, grid)
        self.g, self.g_end = self.sk.start(c), self.sk.start(c + 1)
        self.dp_next = c

    def next(self):
        if self.dp_next < self.dp_tiles:
            t = self.dp_next
            self.dp_next += self.G
            return t, 0, self.KS
        if self.g < self.g_end:
            lt = self.g // self.KS
            k0 = self.g % self.KS
            k1 = min(self.KS, k0 + (self.g_end - self.g))
            self.g += k1 - k0
            return self.dp_tiles + lt, k0, k1
        return None

    def is_split_tile(self, tile):
        return tile >= self.dp_tiles

    def sk_begin(self):
        return self.sk.start(self.cta)

    def tile_begin(self, tile):
        return (tile - self.dp_tiles) * self.KS

    def ranges_cover_a_tile(self):
        return self.sk.W // self.G >= self.KS


def simulate(num_tiles, ks, grid):
    cover = {}
    counters = {}
    partial_slots = {}
    pairs = set()
    for c in range(grid):
        s = Schedule(num_tiles, ks, grid, c)
        seen_split = False
        while (seg := s.next()) is not None:
            tile, k0, k1 = seg
            assert 0 <= tile < num_tiles and 0 <= k0 < k1 <= ks
            cover.setdefault(tile, []).append((k0, k1, c))
            if k0 != 0 or k1 != ks:
                seen_split = True
                assert s.is_split_tile(tile)
                tb = s.tile_begin(tile)
                slot = 0 if s.sk_begin() >= tb else 1
                key = (c, slot)
                assert key not in partial_slots, f"CTA {c} reuses partial slot {slot}"
                partial_slots[key] = tile
                cf, cl = s.sk.cta_of(tb), s.sk.cta_of(tb + ks - 1)
                assert cf <= c <= cl
                counters.setdefault((tile, cf), []).append(k1 - k0)
                # the summing CTA walks cf..cl and skips empty ranges: the set it reads must
                # be exactly the set of CTAs that stored a partial of this tile
                readers = [x for x in range(cf, cl + 1) if s.sk.start(x) != s.sk.start(x + 1)]
                for x in readers:
                    assert s.sk.start(x) < tb + ks and s.sk.start(x + 1) > tb
                if cl == cf + 1 and s.ranges_cover_a_tile():
                    # two-contributor protocol: the tail is the tail owner's first split
                    # segment, stored in slot 0; the head is the head owner's last segment;
                    # counting steps at equal speed, the tail is done before the head starts
                    tail_owner = Schedule(num_tiles, ks, grid, cl)
                    head_owner = Schedule(num_tiles, ks, grid, cf)
                    head_len = tb + ks - tb - (tb + ks - s.sk.start(cl))
                    tail_len = ks - head_len
                    assert tail_owner.sk_begin() >= tb  # slot 0
                    assert head_owner.sk.start(cf + 1) == tb + head_len  # head ends cf's range
                    assert tail_len <= (head_owner.sk.start(cf + 1) - head_owner.sk_begin()) - head_len
                    pairs.add(tile)
            elif not s.is_split_tile(tile):
                assert not seen_split, "whole tile after a split segment"
    for t in range(num_tiles):
        segs = sorted(cover.get(t, []))
        assert segs, f"tile {t} not covered"
        pos = 0
        for k0, k1, _ in segs:
            assert k0 == pos, f"tile {t}: gap or overlap at {pos}"
            pos = k1
        assert pos == ks
    for (tile, cf), parts in counters.items():
        assert sum(parts) == ks, (tile, parts)
    return cover


@pytest.mark.parametrize("num_tiles,ks,grid", list(itertools.product(
    [1, 2, 3, 47, 48, 147, 148, 149, 240, 295, 296, 297, 420, 448, 1536, 3000],
    [1, 2, 7, 16, 56, 128],
    [1, 2, 3, 132, 148])))
def test_schedule_covers_and_protocol_holds(num_tiles, ks, grid):
    simulate(num_tiles, ks, grid)


def test_cta_of_inverts_start():
    for W, G in itertools.product([1, 5, 56, 1000, 13440], [1, 3, 148]):
        sk = StreamK(W, G)
        for g in range(W):
            c = sk.cta_of(g)
            assert sk.start(c) <= g < sk.start(c + 1), (W, G, g, c)


def test_whole_tiles_are_a_multiple_of_the_grid():
    for n, G in itertools.product([1, 148, 296, 297, 444, 1000, 4096], [1, 148]):
        s = Schedule(n, 56, G, 0)
        if G // 2 <= n <= G and 2 * n >= G:
            assert s.dp_tiles == n  # one whole tile per CTA, nothing split
            continue
        assert s.dp_tiles % G == 0 and 0 <= n - s.dp_tiles
        if n > 2 * G:
            assert G <= n - s.dp_tiles < 2 * G


def test_few_tiles_run_whole_or_split_by_count():
    G = 148
    for n in range(1, 2 * G + 1):
        s = Schedule(n, 56, G, 0)
        whole = n <= G and 2 * n >= G
        assert (s.dp_tiles == n) == whole and (s.dp_tiles == 0) == (not whole)
