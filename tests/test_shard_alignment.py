"""Shard alignment, overlap and pack/unpack (CPU).

The alignment cases are the contract of the reference's
``tests/test_shard_compatibility.py:32-347`` (pair form, single-shard overlap form,
``pack_for`` / ``tensors_from_flat`` round trip); the property tests check the
refinement against a dense oracle on random factorisations.
"""
import random

import pytest
import torch

from weightbridge_b200 import WeightData
from weightbridge_b200.core.binding import bind, pack_into, unpack_from, strided
from weightbridge_b200.core.shard import (_nested, align_shards, box_copies, box_copy,
                                          check_shard_compatibility, coalesce)

# (sender, receiver, expected aligned sender, expected aligned receiver); None = incompatible
CASES = {
    "same_dims": ([(0, 4, 4), (0, 6, 6)], [(2, 3, 4), (1, 5, 6)],
                  [(0, 4, 4), (0, 6, 6)], [(2, 3, 4), (1, 5, 6)]),
    "sender_flat_receiver_split": ([(0, 24, 24)], [(0, 4, 4), (0, 6, 6)],
                                   [(0, 4, 4), (0, 6, 6)], [(0, 4, 4), (0, 6, 6)]),
    "receiver_flat_sender_split": ([(0, 4, 4), (0, 6, 6)], [(0, 24, 24)],
                                   [(0, 4, 4), (0, 6, 6)], [(0, 4, 4), (0, 6, 6)]),
    "sender_flat_full_rows": ([(6, 12, 24)], [(0, 4, 4), (0, 6, 6)],
                              [(1, 2, 4), (0, 6, 6)], [(0, 4, 4), (0, 6, 6)]),
    "sender_flat_single_row": ([(1, 5, 24)], [(0, 4, 4), (0, 6, 6)],
                               [(0, 1, 4), (1, 5, 6)], [(0, 4, 4), (0, 6, 6)]),
    "receiver_flat_single_row": ([(0, 4, 4), (0, 6, 6)], [(7, 11, 24)],
                                 [(0, 4, 4), (0, 6, 6)], [(1, 2, 4), (1, 5, 6)]),
    "multi_level_split": ([(4, 8, 24)], [(0, 2, 2), (0, 3, 3), (0, 4, 4)],
                          [(0, 1, 2), (1, 2, 3), (0, 4, 4)], [(0, 2, 2), (0, 3, 3), (0, 4, 4)]),
    "both_partial": ([(1, 3, 4), (2, 5, 6)], [(2, 4, 4), (0, 4, 6)],
                     [(1, 3, 4), (2, 5, 6)], [(2, 4, 4), (0, 4, 6)]),
    "sender_3d_receiver_1d": ([(0, 2, 2), (0, 3, 3), (0, 4, 4)], [(0, 24, 24)],
                              [(0, 2, 2), (0, 3, 3), (0, 4, 4)], [(0, 2, 2), (0, 3, 3), (0, 4, 4)]),
    "single_dim": ([(2, 7, 10)], [(4, 9, 10)], [(2, 7, 10)], [(4, 9, 10)]),
    "4x6_vs_2x4x3": ([(0, 4, 4), (0, 6, 6)], [(0, 2, 2), (0, 4, 4), (0, 3, 3)],
                     [(0, 2, 2)] * 3 + [(0, 3, 3)], [(0, 2, 2)] * 3 + [(0, 3, 3)]),
    "4x6_vs_2x12": ([(0, 4, 4), (0, 6, 6)], [(0, 2, 2), (0, 12, 12)],
                    [(0, 2, 2), (0, 2, 2), (0, 6, 6)], [(0, 2, 2), (0, 2, 2), (0, 6, 6)]),
    "3x2x4_vs_6x4": ([(0, 3, 3), (0, 2, 2), (0, 4, 4)], [(0, 6, 6), (0, 4, 4)],
                     [(0, 3, 3), (0, 2, 2), (0, 4, 4)], [(0, 3, 3), (0, 2, 2), (0, 4, 4)]),
    "3x2x4_vs_6x4_partial": ([(1, 3, 3), (0, 2, 2), (1, 3, 4)], [(2, 4, 6), (0, 4, 4)],
                             [(1, 3, 3), (0, 2, 2), (1, 3, 4)], [(1, 2, 3), (0, 2, 2), (0, 4, 4)]),
    "8x3_vs_4x6": ([(2, 6, 8), (0, 3, 3)], [(0, 4, 4), (0, 6, 6)],
                   [(1, 3, 4), (0, 2, 2), (0, 3, 3)], [(0, 4, 4), (0, 2, 2), (0, 3, 3)]),
    "2x2x6_vs_4x3x2": ([(0, 2, 2), (0, 2, 2), (0, 6, 6)], [(0, 4, 4), (0, 3, 3), (0, 2, 2)],
                       [(0, 2, 2), (0, 2, 2), (0, 3, 3), (0, 2, 2)],
                       [(0, 2, 2), (0, 2, 2), (0, 3, 3), (0, 2, 2)]),
    "1d_vs_4d": ([(0, 48, 48)], [(0, 2, 2), (0, 3, 3), (0, 2, 2), (0, 4, 4)],
                 [(0, 2, 2), (0, 3, 3), (0, 2, 2), (0, 4, 4)], None),
    "1d_partial_vs_4d": ([(0, 24, 48)], [(0, 2, 2), (0, 3, 3), (0, 2, 2), (0, 4, 4)],
                         [(0, 1, 2), (0, 3, 3), (0, 2, 2), (0, 4, 4)], None),
    "4x6_vs_2x4x3_partial": ([(0, 4, 4), (0, 6, 6)], [(0, 2, 2), (2, 4, 4), (0, 3, 3)],
                             [(0, 2, 2)] * 3 + [(0, 3, 3)],
                             [(0, 2, 2), (1, 2, 2), (0, 2, 2), (0, 3, 3)]),
    "mixed_partial_full": ([(0, 4, 4), (0, 6, 6)], [(0, 2, 2), (6, 12, 12)],
                           [(0, 2, 2), (0, 2, 2), (0, 6, 6)], [(0, 2, 2), (1, 2, 2), (0, 6, 6)]),
}

INCOMPATIBLE = {
    "spans_multiple_rows": ([(5, 13, 24)], [(0, 4, 4), (0, 6, 6)]),
    "not_divisible": ([(0, 10, 12)], [(0, 3, 3), (0, 4, 4)]),
    "transposed": ([(0, 4, 4), (0, 3, 3)], [(0, 3, 3), (0, 4, 4)]),
    "coprime_first": ([(0, 3, 3), (0, 8, 8)], [(0, 4, 4), (0, 6, 6)]),
    "receiver_multi_rows": ([(0, 3, 3), (0, 4, 4)], [(1, 11, 12)]),
    "inner_not_rectangular": ([(2, 6, 8), (0, 3, 3)], [(0, 4, 4), (1, 5, 6)]),
    "nonrect_3d": ([(10, 20, 24)], [(0, 2, 2), (0, 3, 3), (0, 4, 4)]),
    "deep_not_divisible": ([(0, 10, 10), (0, 3, 3)], [(0, 6, 6), (0, 5, 5)]),
    "partial_receiver_complex": ([(1, 3, 3), (0, 2, 2), (1, 3, 4)], [(2, 5, 6), (0, 4, 4)]),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_alignment_pair_form(name):
    s, r, exp_s, exp_r = CASES[name]
    res = check_shard_compatibility(s, r)
    assert res is not None
    got_s, got_r = res
    assert got_s == exp_s
    if exp_r is not None:
        assert got_r == exp_r
    assert [w for *_, w in got_s] == [w for *_, w in got_r]


@pytest.mark.parametrize("name", sorted(INCOMPATIBLE))
def test_alignment_incompatible(name):
    s, r = INCOMPATIBLE[name]
    assert check_shard_compatibility(s, r) is None
    assert align_shards(s, r) is None


def test_five_tuple_form():
    assert align_shards([(1, 5, 24)], [(0, 4, 4), (0, 6, 6)]) == [(0, 1, 0, 4, 4), (1, 5, 0, 6, 6)]


def test_trailing_unit_dims_absorbed():
    assert check_shard_compatibility([(0, 4, 4)], [(0, 4, 4), (0, 1, 1)]) == (
        [(0, 4, 4), (0, 1, 1)], [(0, 4, 4), (0, 1, 1)])


def _meta(shard, dtype=torch.float32):
    return WeightData({"weight": {"shard": shard, "dtype": dtype}})


def test_overlap_single_shard_form():
    ov = WeightData.compute_overlap(_meta([(1, 3, 4), (0, 6, 6)]), _meta([(2, 4, 4), (2, 5, 6)]))
    assert "weight" in ov.meta_dict
    assert ov["weight"]["shard"] == [(2, 3, 4), (2, 5, 6)]


def test_overlap_disjoint_is_empty():
    ov = WeightData.compute_overlap(_meta([(0, 2, 4), (0, 6, 6)]), _meta([(2, 4, 4), (0, 6, 6)]))
    assert len(ov.meta_dict) == 0 and not ov


def test_overlap_incompatible_raises():
    with pytest.raises(ValueError):             # different logical sizes
        WeightData.compute_overlap(_meta([(0, 24, 24)]), _meta([(0, 5, 5), (0, 5, 5)]))


def test_cross_factorisations_are_refused():
    """4 x 6 against 6 x 4 of the same 24 elements: not refinements of one shape, which in a
    real layout means a transposed or mis-declared tensor, so the overlap is an error."""
    with pytest.raises(ValueError, match="refinements of one shape"):
        WeightData.compute_overlap(_meta([(0, 4, 4), (1, 6, 6)]), _meta([(0, 6, 6), (0, 4, 4)]))


def test_overlap_cuts_a_range_through_rows_into_rectangles():
    """A flat range that starts and ends inside rows of the other side's 4 x 6 box has no
    single rectangular overlap; it is cut at the row boundaries (the pair-form check keeps
    the reference's answer, no common refinement)."""
    assert check_shard_compatibility([(5, 13, 24)], [(0, 4, 4), (0, 6, 6)]) is None
    ov = WeightData.compute_overlap(_meta([(5, 13, 24)]), _meta([(0, 4, 4), (0, 6, 6)]))
    assert ov.shards("weight") == [[(0, 1, 4), (5, 6, 6)], [(1, 2, 4), (0, 6, 6)], [(2, 3, 4), (0, 1, 6)]]
    assert ov.total_nbytes() == 8 * 4
    flat = torch.arange(24, dtype=torch.float32)
    s = _meta([(5, 13, 24)])
    packed = WeightData.pack_for(s, {"weight": flat[5:13]}, ov)
    got = torch.full((4, 6), -1.0)
    unpack_from(bind(_meta([(0, 4, 4), (0, 6, 6)]), {"weight": got}), ov, packed)
    exp = torch.full((24,), -1.0)
    exp[5:13] = flat[5:13]
    assert torch.equal(got.reshape(-1), exp)


def test_pack_for_roundtrip():
    shard = [(0, 4, 4), (0, 6, 6)]
    s = _meta(shard)
    ov = WeightData.compute_overlap(s, s)
    t = torch.arange(24, dtype=torch.float32).reshape(4, 6)
    packed = WeightData.pack_for(s, {"weight": t}, ov)
    assert packed.dtype == torch.uint8 and packed.numel() == 24 * 4
    assert torch.equal(ov.tensors_from_flat(packed)["weight"], t)


def test_json_roundtrip_and_accounting():
    wd = WeightData({
        "a": {"shard": [(0, 2, 4), (0, 3, 3)], "dtype": "bfloat16"},
        "b": {"shard": [[(0, 1, 4)], [(2, 5, 8)]], "dtype": torch.float32},
    })
    again = WeightData(bytes(wd))
    assert again == wd
    assert again.dtype("a") == torch.bfloat16
    # multi-shard entry = disjoint union: 1 + 3 elements
    assert wd.numel("b") == 4
    assert wd.total_nbytes() == 6 * 2 + 4 * 4
    intv = [(s, e, n) for s, e, n, _, _ in wd.iter_with_intv()]
    assert intv == [(0, 12, "a"), (12, 28, "b")]


def test_invalid_shards_rejected():
    with pytest.raises(ValueError):
        WeightData({"x": {"shard": [(3, 2, 4)], "dtype": "float32"}})
    with pytest.raises(ValueError):
        WeightData({"x": {"shard": [], "dtype": "float32"}})


def test_bridge_does_not_mutate_callers_dict():
    s = _meta([(0, 4, 4), (0, 6, 6)])
    t = torch.randn(4, 6)
    tensors = {"weight": t, "other": torch.zeros(3)}
    bridge = s(tensors)
    ov = WeightData.compute_overlap(s, _meta([(1, 3, 4), (0, 6, 6)]))
    chunk = bridge[{7: ov}][7]
    assert set(tensors) == {"weight", "other"} and tensors["weight"] is t
    r_tensor = torch.zeros(2, 6)
    _meta([(1, 3, 4), (0, 6, 6)])({"weight": r_tensor})[{7: ov}] = {7: chunk}
    assert torch.equal(r_tensor, t[1:3])


def test_coalesce():
    assert coalesce([4, 6], [6, 1], [6, 1]) == ([24], [1], [1])
    assert coalesce([4, 6], [12, 1], [6, 1]) == ([4, 6], [12, 1], [6, 1])
    assert coalesce([1, 3, 1, 5], [99, 5, 7, 1], [0, 5, 3, 1]) == ([15], [1], [1])


# ----------------------------------------------------------------------------------------
# property tests: random factorisations against a dense oracle
# ----------------------------------------------------------------------------------------

def _random_box(rng, shape):
    box = []
    for w in shape:
        l = rng.randrange(w)
        r = rng.randrange(l + 1, w + 1)
        box.append((l, r, w))
    return box


def _merge(box, i):
    """Merge dims i, i+1 of a box if the result is still a box; else None."""
    (l0, r0, w0), (l1, r1, w1) = box[i], box[i + 1]
    if l1 == 0 and r1 == w1:
        m = (l0 * w1, r0 * w1, w0 * w1)
    elif r0 == l0 + 1:
        m = (l0 * w1 + l1, l0 * w1 + r1, w0 * w1)
    else:
        return None
    return box[:i] + [m] + box[i + 2:]


def _split(box, i, a):
    l, r, w = box[i]
    b = w // a
    if l % b == 0 and r % b == 0:
        parts = [(l // b, r // b, a), (0, b, b)]
    elif l // b == (r - 1) // b:
        row = l // b
        parts = [(row, row + 1, a), (l - row * b, r - row * b, b)]
    else:
        return None
    return box[:i] + parts + box[i + 1:]


def _reshape_randomly(rng, box, steps=3):
    for _ in range(steps):
        if rng.random() < 0.5 and len(box) > 1:
            m = _merge(box, rng.randrange(len(box) - 1))
            if m is not None:
                box = m
        else:
            i = rng.randrange(len(box))
            w = box[i][2]
            divs = [d for d in range(2, w) if w % d == 0]
            if divs:
                s = _split(box, i, rng.choice(divs))
                if s is not None:
                    box = s
    return box


def _logical_region(nd_box):
    return tuple(slice(l, r) for l, r, _ in nd_box)


@pytest.mark.parametrize("seed", range(60))
def test_box_copy_matches_dense_oracle(seed):
    rng = random.Random(seed)
    shape = [rng.choice([2, 4, 6, 8, 12]) for _ in range(rng.choice([1, 2, 3]))]
    logical = torch.arange(1, 1 + torch.tensor(shape).prod().item(), dtype=torch.float64).reshape(shape)
    sb, rb = _random_box(rng, shape), _random_box(rng, shape)
    s_repr, r_repr = _reshape_randomly(rng, sb), _reshape_randomly(rng, rb)
    src = logical[_logical_region(sb)].contiguous()
    dst = torch.zeros([r - l for l, r, _ in rb], dtype=torch.float64)
    try:
        bc = box_copy(s_repr, r_repr)
    except ValueError:
        # incompatible factorisations are allowed to fail, but the same shapes must align
        assert s_repr != r_repr or False
        return
    inter = [(max(a[0], b[0]), min(a[1], b[1])) for a, b in zip(sb, rb)]
    expect = dst.clone()
    if all(lo < hi for lo, hi in inter):
        sub = logical[tuple(slice(lo, hi) for lo, hi in inter)]
        expect[tuple(slice(lo - b[0], hi - b[0]) for (lo, hi), b in zip(inter, rb))] = sub
    if bc is None:
        assert torch.equal(expect, dst)
        return
    strided(dst, bc.dst_offset, bc.extents, bc.dst_strides).copy_(
        strided(src, bc.src_offset, bc.extents, bc.src_strides))
    assert torch.equal(dst, expect)


@pytest.mark.parametrize("seed", range(20))
def test_pack_unpack_multi_receiver(seed):
    """Sender holds a column split, receivers a row split: pack per receiver, unpack."""
    rng = random.Random(seed)
    rows, cols = rng.choice([4, 8]), rng.choice([6, 12])
    full = torch.randn(rows, cols)
    c = rng.randrange(1, cols)
    senders = [WeightData({"w": {"shard": [(0, rows, rows), (0, c, cols)], "dtype": "float32"}}),
               WeightData({"w": {"shard": [(0, rows, rows), (c, cols, cols)], "dtype": "float32"}})]
    s_tensors = [full[:, :c].contiguous(), full[:, c:].contiguous()]
    r0 = rng.randrange(1, rows)
    receivers = [WeightData({"w": {"shard": [(0, r0 * cols, rows * cols)], "dtype": "float32"}}),
                 WeightData({"w": {"shard": [(r0 * cols, rows * cols, rows * cols)], "dtype": "float32"}})]
    r_tensors = [torch.zeros(r0 * cols), torch.zeros((rows - r0) * cols)]
    for si, sm in enumerate(senders):
        b = bind(sm, {"w": s_tensors[si]})
        for ri, rm in enumerate(receivers):
            ov = WeightData.compute_overlap(sm, rm)
            if not ov:
                continue
            buf = torch.empty(ov.total_nbytes(), dtype=torch.uint8)
            pack_into(b, ov, buf)
            unpack_from(bind(rm, {"w": r_tensors[ri]}), ov, buf)
    assert torch.equal(torch.cat(r_tensors), full.reshape(-1))


@pytest.mark.parametrize("seed", range(80))
def test_box_copies_cut_ranges_against_dense_oracle(seed):
    """A flat range (an FSDP-style row range) against a partial N-d box of the same tensor,
    either side as the source: the pieces write every element of the intersection exactly
    once, with the right value, and nothing else."""
    import math
    rng = random.Random(seed)
    shape = [rng.choice([2, 3, 4, 6]) for _ in range(rng.choice([2, 3]))]
    n = math.prod(shape)
    a = rng.randrange(n)
    b = rng.randrange(a + 1, n + 1)
    flat, box = [(a, b, n)], _random_box(rng, shape)
    logical = torch.arange(1, n + 1, dtype=torch.float64)
    in_box = logical.reshape(shape)[_logical_region(box)]          # values = logical index + 1
    in_range = ((in_box - 1) >= a) & ((in_box - 1) < b)
    if rng.random() < 0.5:                                          # flat source, box destination
        src, dst = logical[a:b].clone(), torch.zeros(in_box.shape, dtype=torch.float64)
        bcs = box_copies(flat, box)
        expect = torch.where(in_range, in_box, torch.zeros_like(in_box))
    else:                                                           # box source, flat destination
        src, dst = in_box.contiguous(), torch.zeros(b - a, dtype=torch.float64)
        bcs = box_copies(box, flat)
        full = torch.zeros(n, dtype=torch.float64)
        full[(in_box[in_range] - 1).long()] = in_box[in_range]
        expect = full[a:b]
    count = torch.zeros_like(dst)
    for bc in bcs:
        strided(dst, bc.dst_offset, bc.extents, bc.dst_strides).copy_(
            strided(src, bc.src_offset, bc.extents, bc.src_strides))
        strided(count, bc.dst_offset, bc.extents, bc.dst_strides).add_(1)
    assert torch.equal(dst, expect)
    assert (count <= 1).all() and int(count.sum()) == int(in_range.sum())


@pytest.mark.parametrize("seed", range(300))
def test_box_copies_random_factorisations_against_dense_oracle(seed):
    """Two partial boxes of one tensor, each re-factorised at random: box_copies returns
    pieces for every pair of refinements of one shape (and whenever box_copy aligns), which
    write exactly the intersection, once per element, and agrees with box_copy on whether
    they intersect; cross factorisations that box_copy refuses stay refused."""
    rng = random.Random(1000 + seed)
    shape = [rng.choice([2, 3, 4, 6, 8]) for _ in range(rng.choice([1, 2, 3]))]
    logical = torch.arange(1, 1 + torch.tensor(shape).prod().item(), dtype=torch.float64).reshape(shape)
    sb, rb = _random_box(rng, shape), _random_box(rng, shape)
    s_repr, r_repr = _reshape_randomly(rng, sb, steps=4), _reshape_randomly(rng, rb, steps=4)
    try:
        single = box_copy(s_repr, r_repr)
        single_ok = True
    except ValueError:
        single_ok = False
    try:
        bcs = box_copies(s_repr, r_repr)     # every pair of refinements of one shape aligns
    except ValueError:
        assert not single_ok and not _nested(s_repr, r_repr)
        return
    src = logical[_logical_region(sb)].contiguous()
    dst = torch.zeros([r - l for l, r, _ in rb], dtype=torch.float64)
    count = torch.zeros_like(dst)
    for bc in bcs:
        strided(dst, bc.dst_offset, bc.extents, bc.dst_strides).copy_(
            strided(src, bc.src_offset, bc.extents, bc.src_strides))
        strided(count, bc.dst_offset, bc.extents, bc.dst_strides).add_(1)
    inter = [(max(a[0], b[0]), min(a[1], b[1])) for a, b in zip(sb, rb)]
    expect = torch.zeros_like(dst)
    if all(lo < hi for lo, hi in inter):
        sub = logical[tuple(slice(lo, hi) for lo, hi in inter)]
        expect[tuple(slice(lo - b[0], hi - b[0]) for (lo, hi), b in zip(inter, rb))] = sub
    assert torch.equal(dst, expect)
    assert (count <= 1).all() and int(count.sum()) == int((expect != 0).sum())
    if single_ok:
        assert (single is None) == (not bcs)
