"""Host-side residency and read planning through the C ABI (no GPU needed):
should_keep_resident (persistent.rs:468, its test at :490-495) and
build_layer_read_plan (layer_read.rs:50-132, its tests at :134-200), restated
case for case, plus the refusals and the limits of both coalescing rules."""
import pytest

from ramforge_b200 import RfError, layer_read_plan, should_keep_resident

KIB, MIB = 1024, 1024 * 1024
U64_MAX = (1 << 64) - 1


def test_persistent_policy_uses_resident_bytes_and_is_overflow_safe():
    assert should_keep_resident(250, 1000)
    assert not should_keep_resident(251, 1000)
    assert not should_keep_resident(U64_MAX, U64_MAX)
    assert should_keep_resident(U64_MAX // 4, U64_MAX)


def test_adjacent_and_arbitrarily_ordered_tensors_coalesce():
    ranges, placed, tot = layer_read_plan([(108, 4), (100, 4), (104, 4)])
    assert tot["logical_tensor_count"] == 3
    assert len(ranges) == 1
    assert ranges[0]["file_offset"] == 100 and ranges[0]["byte_length"] == 12 and ranges[0]["gap_bytes"] == 0
    assert ranges[0]["tensors"] == [1, 2, 0]


def test_small_gap_is_bounded_overhead_not_logical_data():
    ranges, placed, tot = layer_read_plan([(100, 8), (116, 8)])
    assert len(ranges) == 1
    assert tot["logical_bytes"] == 16 and tot["physical_bytes"] == 24 and tot["gap_bytes"] == 8
    assert placed[1]["offset_in_range"] == 16


def test_reusable_buffer_requires_multiple_fully_grouped_ranges():
    gap = 4 * KIB + 1
    ranges, _, tot = layer_read_plan([(0, 4), (4, 4), (8 + gap, 4), (12 + gap, 4)])
    assert len(ranges) == 2
    assert tot["reusable_group_buffer_bytes"] == 8
    _, _, tot = layer_read_plan([(0, 4), (gap, 4)])
    assert tot["reusable_group_buffer_bytes"] == 0


def test_gap_and_span_limits_are_inclusive():
    assert len(layer_read_plan([(0, 4), (4 + 4 * KIB, 4)])[0]) == 1  # a gap of exactly 4 KiB joins
    assert len(layer_read_plan([(0, 4), (5 + 4 * KIB, 4)])[0]) == 2
    assert len(layer_read_plan([(0, 32 * MIB), (32 * MIB, 32 * MIB)])[0]) == 1  # a span of exactly 64 MiB joins
    assert len(layer_read_plan([(0, 32 * MIB), (32 * MIB, 32 * MIB + 1)])[0]) == 2


def test_overlap_and_overflow_are_refused():
    with pytest.raises(RfError, match="INVAL"):
        layer_read_plan([(100, 8), (104, 8)])
    with pytest.raises(RfError, match="INVAL"):
        layer_read_plan([(U64_MAX - 2, 8)])


def test_llama_layer_tensors_coalesce_into_one_read():
    # nine tensors of a GGUF layer, 32-byte aligned with small gaps: one read
    sizes = [16384, 9437184, 2359296, 2359296, 9437184, 16384, 33030144, 33030144, 33030144]
    ext, off = [], 1000
    for b in sizes:
        ext.append((off, b))
        off = (off + b + 31) // 32 * 32 + 32
    ranges, _, tot = layer_read_plan(ext)
    assert tot["logical_bytes"] == sum(sizes)
    assert tot["physical_bytes"] == sum(r["byte_length"] for r in ranges)
    assert all(r["byte_length"] <= 64 * MIB for r in ranges)
    assert [i for r in ranges for i in r["tensors"]] == list(range(9))
