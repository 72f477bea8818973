"""The balanced row-group schedule of the decode kernel's projection phases, checked on the CPU.

A restatement of the integer arithmetic of ``gemv_geom`` (decode_kernel.cuh) and of the host's
``split_kinds`` rule (engine.cu): tile_shape's segment count, whole-group ranges per CTA slot, and, for
the phases the rule splits, the even (group, segment) ranges with their lead (tail part) and tail (head
part) pieces.  For every model shape the kernel serves (Gemma3-1B fp32, 4B and 27B bf16, a 4B rank at
TP=2, the test shapes) every tile must be streamed exactly once, every split group must have exactly
two owners -- adjacent slots, one head part [0, s) and one tail part [s, nseg) -- and the largest share
must not exceed the even share by more than one tile.
"""

from __future__ import annotations

import pytest

STAGE_BYTES = 36864
CTAS = 148


def tile_shape(kp: int, esz: int, pair: bool) -> tuple[int, int]:
    """(rows per group, segments) of decode.cuh's tile_shape."""
    rps = 8 * (2 if esz == 2 else 1)
    n = max(1, -(-kp * rps * (2 if pair else 1) * esz // STAGE_BYTES))
    while kp % n or (kp // n) % 8:
        n += 1
    return rps, n


def splits(groups: int, nseg: int, G: int) -> bool:
    """engine.cu split_kinds for one phase."""
    U = groups * nseg
    if nseg < 2 or U // G < nseg or U * G >= 1 << 31:
        return False
    return -(-groups // G) * nseg - -(-U // G) >= 2


def schedule(groups: int, nseg: int, G: int, split: bool) -> list[dict]:
    """Per slot: whole groups and split pieces, as gemv_geom computes them."""
    out = []
    for slot in range(G):
        g0, g1 = groups * slot // G, groups * (slot + 1) // G
        s = {"full": (g0, g1 - g0), "lead": None, "tail": None}
        if split:
            U = groups * nseg
            u0, u1 = U * slot // G, U * (slot + 1) // G
            ga, sa = divmod(u0, nseg)
            gb, sb = divmod(u1, nseg)
            full_g0 = ga + 1 if sa else ga
            s["full"] = (full_g0, gb - full_g0)
            s["lead"] = (ga, sa) if sa else None  # segments [sa, nseg) of group ga: part 1
            s["tail"] = (gb, sb) if sb else None  # segments [0, sb) of group gb: part 0
        out.append(s)
    return out


def phases(hidden: int, inter: int, hq: int, hkv: int, hd: int, esz: int) -> list[tuple[str, int, int, bool]]:
    pad = lambda k: -(-k // 128) * 128  # noqa: E731
    return [("QKV", (hq + 2 * hkv) * hd, pad(hidden), False), ("O", hidden, pad(hq * hd), False),
            ("GU", inter, pad(hidden), True), ("D", hidden, pad(inter), False)]


SHAPES = {
    "gemma3-1b f32": (1152, 6912, 4, 1, 256, 4),
    "gemma3-4b bf16": (2560, 10240, 8, 4, 256, 2),
    "gemma3-27b bf16": (5376, 21504, 32, 16, 128, 2),
    "gemma3-4b bf16 tp2 rank": (2560, 5120, 4, 2, 256, 2),
    "test 2560x4096 bf16": (2560, 4096, 4, 1, 256, 2),
    "test 1536x2560 bf16": (1536, 2560, 4, 1, 256, 2),
}
EXPECTED = {  # phases the rule splits (bf16 kernels only)
    "gemma3-1b f32": set(),
    "gemma3-4b bf16": {"GU", "D"},
    "gemma3-27b bf16": {"QKV", "O", "GU", "D"},
    "gemma3-4b bf16 tp2 rank": {"GU", "D"},
    "test 2560x4096 bf16": {"D"},
    "test 1536x2560 bf16": {"GU"},
}


@pytest.mark.parametrize("shape", sorted(SHAPES))
def test_schedule_covers_every_tile_once(shape: str) -> None:
    hidden, inter, hq, hkv, hd, esz = SHAPES[shape]
    split_phases = set()
    for name, n, kp, pair in phases(hidden, inter, hq, hkv, hd, esz):
        rps, nseg = tile_shape(kp, esz, pair)
        groups = -(-n // rps)
        split = esz == 2 and splits(groups, nseg, CTAS)
        if split:
            split_phases.add(name)
        sched = schedule(groups, nseg, CTAS, split)
        seen: dict[tuple[int, int], int] = {}
        owners: dict[int, list[tuple[int, int]]] = {}
        for slot, s in enumerate(sched):
            g0, nf = s["full"]
            assert nf >= 0
            tiles = 0
            for g in range(g0, g0 + nf):
                for sg in range(nseg):
                    seen[(g, sg)] = seen.get((g, sg), 0) + 1
                    tiles += 1
            if s["lead"]:
                g, sa = s["lead"]
                for sg in range(sa, nseg):
                    seen[(g, sg)] = seen.get((g, sg), 0) + 1
                    tiles += 1
                owners.setdefault(g, []).append((slot, 1))
            if s["tail"]:
                g, sb = s["tail"]
                for sg in range(sb):
                    seen[(g, sg)] = seen.get((g, sg), 0) + 1
                    tiles += 1
                owners.setdefault(g, []).append((slot, 0))
            if split:
                assert tiles <= -(-groups * nseg // CTAS), (name, slot, tiles)
        assert seen == {(g, sg): 1 for g in range(groups) for sg in range(nseg)}, name
        for g, own in owners.items():
            assert sorted(p for _s, p in own) == [0, 1], (name, g, own)
            head = next(s for s, p in own if p == 0)
            tail = next(s for s, p in own if p == 1)
            assert tail == head + 1, (name, g, own)  # the boundary index is the head owner's slot
    assert split_phases == EXPECTED[shape]


def test_gemma3_1b_needs_no_split() -> None:
    """Even without the bf16-only restriction the rule splits no phase of Gemma3-1B fp32: its whole groups
    are already within one tile of the even share."""
    for name, n, kp, pair in phases(*SHAPES["gemma3-1b f32"]):
        rps, nseg = tile_shape(kp, 4, pair)
        assert not splits(-(-n // rps), nseg, CTAS), name
