"""The FP8 expert record layout and its index.json schema (host-only checks).

The record format rules of docs/dev/format.md:37-76: parts at 256-byte
(PART_ALIGN) offsets in the schema's order, record stride a multiple of 4096
(ALIGN), zero padding; the C layout function agrees with a restatement of
those rules here."""
import pytest

from homelab_b200 import SCALE_128X128, SCALE_1X128
from homelab_b200.convert import LAYOUT_TAGS, record_layout, record_schema


def _restated(hidden, inter, layout):
    up = lambda v, a: (v + a - 1) // a * a  # noqa: E731
    sb = lambda n, k: ((n + 127) // 128 if layout == SCALE_128X128 else n) * ((k + 127) // 128) * 4  # noqa: E731
    o, offs = 0, []
    for nbytes in (inter * hidden, inter * hidden, hidden * inter, sb(inter, hidden), sb(inter, hidden),
                   sb(hidden, inter)):
        offs.append(o)
        o = up(o + nbytes, 256)
    return offs, up(o, 4096)


@pytest.mark.parametrize("hidden,inter", [(2048, 768), (4096, 1408), (4096, 2048), (256, 144), (4096, 16)])
@pytest.mark.parametrize("layout", [SCALE_128X128, SCALE_1X128])
def test_layout_follows_the_format_rules(hidden, inter, layout):
    g, stride = record_layout(hidden, inter, layout)
    offs, want_stride = _restated(hidden, inter, layout)
    got = [g.gate_weight, g.up_weight, g.down_weight, g.gate_scale, g.up_scale, g.down_scale]
    assert got == offs and stride == want_stride
    assert stride % 4096 == 0 and all(o % 256 == 0 for o in got)
    parts, s2 = record_schema(hidden, inter, layout)
    assert s2 == stride
    assert [p["name"] for p in parts] == ["gate.weight", "up.weight", "down.weight", "gate.weight_scale",
                                          "up.weight_scale", "down.weight_scale"]
    ends = sorted((p["offset"], p["offset"] + p["nbytes"]) for p in parts)
    assert all(a[1] <= b[0] for a, b in zip(ends, ends[1:])) and ends[-1][1] <= stride
    assert LAYOUT_TAGS[layout].startswith("fp8-e4m3-b")


def test_layout_rejects_bad_shapes():
    from homelab_b200._lib import OombError
    with pytest.raises(OombError):
        record_layout(2048, 770)
    with pytest.raises(OombError):
        record_layout(0, 768)
