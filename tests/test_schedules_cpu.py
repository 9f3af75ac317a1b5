"""Work-partition invariants of the GPU schedules, checked on the CPU over
many shapes through line-for-line Python mirrors of the device index maths:
the stream-K split of the small-M kernel (sk_begin / sk_owner, the segment
walk and the partial-slot rule in cuda-fp8-ampere_b200/csrc/gemv_splitk.cu)
and the CTA-pair tcgen05 kernel's work items (tc_item and n_full in
cuda-fp8-ampere_b200/csrc/gemm_tc.cu). The GPU tests check the results of a
few shapes; these check that every unit of work is done exactly once for all
of them."""
import random

import pytest


def sk_begin(c, U, G):
    return c * U // G


def sk_owner(u, U, G):
    return ((u + 1) * G - 1) // U


def walk(U, G, per_mc, hpt):
    plan = {}
    for c in range(G):
        ub, ue = sk_begin(c, U, G), sk_begin(c + 1, U, G)
        segs, u = [], ub
        while u < ue:
            mcl = u // per_mc
            rem = u - mcl * per_mc
            tile, hs = rem // hpt, rem % hpt
            se = min(ue, u - hs + hpt)
            he = hs + (se - u)
            segs.append((mcl, tile, hs, he, u - hs, ub))
            u = se
        plan[c] = segs
    return plan


@pytest.mark.parametrize("seed", range(40))
def test_streamk_partition_covers_every_unit_once(seed):
    rng = random.Random(seed)
    mchunks, tiles, hpt = rng.randint(1, 3), rng.randint(1, 40), rng.randint(1, 140)
    per_mc = tiles * hpt
    U = per_mc * mchunks
    G = rng.randint(1, min(U, 296))
    plan = walk(U, G, per_mc, hpt)
    seen = [0] * U
    slots = {}
    for c, segs in plan.items():
        for (mc, tile, hs, he, tile_u0, ub) in segs:
            assert 0 <= hs < he <= hpt
            for u in range(tile_u0 + hs, tile_u0 + he):
                seen[u] += 1
            whole = hs == 0 and he == hpt
            if not whole:
                slot = 0 if ub >= tile_u0 else 1
                assert (c, slot) not in slots, "a CTA reuses a partial slot"
                slots[(c, slot)] = (mc, tile)
                # the reader finds this CTA's slot with the same rule
                cf, cl = sk_owner(tile_u0, U, G), sk_owner(tile_u0 + hpt - 1, U, G)
                assert cf <= c <= cl
                assert (0 if sk_begin(c, U, G) >= tile_u0 else 1) == slot
    assert all(v == 1 for v in seen)
    # every partially covered tile: contributors = owner(last) - owner(first) + 1, all of them partial
    for mc in range(mchunks):
        for tile in range(tiles):
            u0 = mc * per_mc + tile * hpt
            cf, cl = sk_owner(u0, U, G), sk_owner(u0 + hpt - 1, U, G)
            parts = [k for k, v in slots.items() if v == (mc, tile)]
            if cf != cl:
                assert len(parts) == cl - cf + 1
            else:
                assert len(parts) == 0


def tc_items(tiles_w, tiles_x, tile_x, n_full):
    """(tw, x0, xw) per work item with splits == 1, as tc_item computes it."""
    ntiles = tiles_w * tiles_x
    nwork = n_full + 2 * (ntiles - n_full)
    items = []
    for wi in range(nwork):
        if wi < n_full:
            tile, xw = wi, tile_x
            x0 = (tile // tiles_w) * tile_x
        else:
            j = wi - n_full
            tile, xw = n_full + (j >> 1), tile_x >> 1
            x0 = (tile // tiles_w) * tile_x + (j & 1) * xw
        items.append((tile % tiles_w, x0, xw))
    return items


@pytest.mark.parametrize("tiles_w,tiles_x", [(16, 16), (43, 8), (8, 10), (112, 16), (1, 1), (74, 2), (5, 15)])
def test_tc_half_tail_items_cover_every_tile_once(tiles_w, tiles_x):
    maxpairs, tile_x = 74, 256
    ntiles = tiles_w * tiles_x
    rem = ntiles % maxpairs
    n_full = ntiles
    if ntiles > maxpairs and rem > 0 and 2 * rem <= maxpairs:
        n_full = ntiles - rem
    cover = {}
    for tw, x0, xw in tc_items(tiles_w, tiles_x, tile_x, n_full):
        for x in range(x0, x0 + xw, 32):
            cover[(tw, x)] = cover.get((tw, x), 0) + 1
    assert len(cover) == tiles_w * tiles_x * (tile_x // 32)
    assert all(v == 1 for v in cover.values())
    nwork = n_full + 2 * (ntiles - n_full)
    # the half-width items of the last round fit in one round of pairs
    if n_full < ntiles:
        assert nwork - (nwork // maxpairs) * maxpairs <= maxpairs and 2 * (ntiles - n_full) <= maxpairs


# ---- decode kernel: column groups per cluster, K split (decode.cu) ----------

def decode_groups(NG, P):
    """cg0 / G of every cluster, as the kernel computes them."""
    return [(pc * NG // P, (pc + 1) * NG // P - pc * NG // P) for pc in range(P)]


@pytest.mark.parametrize("N", [8, 24, 513, 1003, 3584, 4096, 7168, 11008])
@pytest.mark.parametrize("P", [1, 25, 74, 148])
def test_decode_groups_cover_every_column_once(N, P):
    NG = (N + 7) // 8
    P = min(P, NG)
    gs = decode_groups(NG, P)
    sizes = [g for _, g in gs]
    assert sum(sizes) == NG
    assert max(sizes) - min(sizes) <= 1  # balanced to within one group
    nxt = 0
    for cg0, g in gs:
        assert cg0 == nxt
        nxt += g


# ---- fused NVLink gather: per-call counter shares (gemv_splitk.cu) ----------

U_CALL = 1 << 20


def gather_share(i, n):
    return (i + 1) * U_CALL // n - i * U_CALL // n


def test_fused_gather_target_alignment_with_alternating_shapes():
    """Every call adds exactly U to each peer counter whatever its cluster
    count, so after e calls of any mix of shapes the counter equals e * U
    (mod 2^32) and the waiting CTA's target stays aligned."""
    rng = random.Random(3)
    ctr = 0
    for e in range(1, 3000):
        clusters = rng.choice([1, 3, 32, 224, 256, 1000, 16384])
        add = sum(gather_share(i, clusters) for i in range(clusters))
        assert add == U_CALL
        assert all(gather_share(i, clusters) > 0 for i in (0, clusters - 1))
        ctr = (ctr + add) % (1 << 32)
        target = (e * U_CALL) % (1 << 32)
        diff = (ctr - target) % (1 << 32)
        assert diff == 0
