"""The prefill grid planner (host code, no GPU): the cluster segments of a
chunk cover every (query row pair, head) unit's causal key tiles exactly once,
a split unit's second key range starts at or below its first query row (so
every row sees a key in both ranges), the second ranges launch after all
first ranges, and the 10 % rule keeps shallow chunks unsplit."""
import ctypes

import pytest

import lisa_attn

AUTO, NEVER, ALWAYS = 0, 1, 2
QH = 24


def plan(base, rows, sms=148, mode=AUTO):
    lib = lisa_attn.load_library()
    lo = (ctypes.c_uint32 * 96)()
    hi = (ctypes.c_uint32 * 96)()
    unit = (ctypes.c_uint16 * 96)()
    n = lib.lisa_attn_debug_prefill_plan(base, rows, sms, mode, lo, hi, unit, 96)
    assert n > 0, n
    return [(lo[i], hi[i], unit[i] & 0xff, (unit[i] >> 8) & 0xf, bool(unit[i] & 0x1000)) for i in range(n)]


def check(base, rows, segs):
    pairs = (((rows + 127) // 128) + 1) // 2
    by_unit = {}
    for lo, hi, h, qp, split in segs:
        assert 0 <= h < QH and 0 <= qp < pairs
        assert lo < hi
        by_unit.setdefault((qp, h), []).append((lo, hi, split))
    assert len(by_unit) == pairs * QH
    for (qp, h), parts in by_unit.items():
        n = (base + min(qp * 256 + 256, rows) + 127) // 128
        parts.sort()
        assert parts[0][0] == 0 and parts[-1][1] == n, (qp, h, parts, n)
        for a, b in zip(parts, parts[1:]):
            assert a[1] == b[0]
        assert len(parts) in (1, 2)
        assert all(p[2] == (len(parts) == 2) for p in parts)
        if len(parts) == 2:
            assert parts[1][0] * 128 <= base + qp * 256  # every row sees a key in the second range
    # second ranges (lo > 0) only after every first range / whole unit
    firsts = [i for i, s in enumerate(segs) if s[0] == 0]
    seconds = [i for i, s in enumerate(segs) if s[0] > 0]
    if seconds:
        assert max(firsts) < min(seconds)


@pytest.mark.parametrize("mode", [AUTO, NEVER, ALWAYS])
@pytest.mark.parametrize("base,rows", [(0, 1), (0, 7), (0, 512), (512, 512), (1536, 512), (3584, 512),
                                       (3584, 1), (8192, 300), (16384, 512), (32256, 512), (100000, 129),
                                       (262143, 1)])
@pytest.mark.parametrize("sms", [148, 132, 8])
def test_plan_covers_every_unit_once(mode, base, rows, sms):
    segs = plan(base, rows, sms, mode)
    check(base, rows, segs)
    if mode == NEVER:
        assert not any(s[4] for s in segs)


def test_plan_splits_deep_chunks_only():
    # shallow config-2 chunks stay one cluster per unit; deep ones split
    assert not any(s[4] for s in plan(0, 512))
    assert not any(s[4] for s in plan(1536, 512))
    deep = plan(16384, 512)
    assert all(s[4] for s in deep) and len(deep) == 96


def test_plan_rejects_bad_arguments():
    lib = lisa_attn.load_library()
    buf = (ctypes.c_uint32 * 96)()
    u = (ctypes.c_uint16 * 96)()
    assert lib.lisa_attn_debug_prefill_plan(0, 0, 148, AUTO, buf, buf, u, 96) == lisa_attn.EINVAL
    assert lib.lisa_attn_debug_prefill_plan(0, 513, 148, AUTO, buf, buf, u, 96) == lisa_attn.EINVAL
    assert lib.lisa_attn_debug_prefill_plan(0, 512, 148, 9, buf, buf, u, 96) == lisa_attn.EINVAL
    assert lib.lisa_attn_debug_prefill_plan(0, 512, 148, AUTO, buf, buf, u, 95) == lisa_attn.EINVAL
