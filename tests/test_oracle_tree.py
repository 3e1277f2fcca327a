"""The oracle's KD-tree lattice builder and SLAT format against the reference's own tests
(SparseLattice.Test/Lattice/EmbeddingLatticeBuilderTests.cs, SerializerTests.cs) and hand-derived
known answers of EmbeddingLatticeBuilder (Lattice/EmbeddingLatticeBuilder.cs) and
SparseLatticeSerializer (Lattice/SparseLatticeSerializer.cs). CPU only."""
import struct

import numpy as np
import pytest

import oracle

INFO = oracle.TREE_INFO_KEYS


def _rows(entries, total_dims):
    """Dense rows from sparse (dimension, value) lists, as SparseVector would hold them."""
    out = np.zeros((len(entries), total_dims), np.int64)
    for i, ent in enumerate(entries):
        for d, v in ent:
            out[i, d] = v
    return out


def _shape(t, i=0):
    """SerializeTreeShape of the reference tests, from the pre-order flattening; returns (text, next)."""
    if t["kind"][i] == 0:
        return f"L({t['count'][i]})", i + 1
    j = i + 1
    below = above = "null"
    if t["mask"][i] & 1:
        below, j = _shape(t, j)
    if t["mask"][i] & 2:
        above, j = _shape(t, j)
    return f"B({t['dim'][i]},{t['val'][i]},{below},{above})", j


def test_empty_input_is_one_empty_leaf():
    t = oracle.tree_build(np.zeros((0, 10), np.int64))
    assert (t["nodes"], t["leaves"], t["occupants"]) == (1, 1, 0)
    assert t["kind"][0] == 0 and t["count"][0] == 0
    # magic 'SLAT', version 1, leaf tag, count 0
    assert oracle.slat_save(np.zeros((0, 10), np.int64), np.zeros(0, np.int32)) == \
        struct.pack("<IHBi", 0x544C4153, 1, 0, 0)


def test_single_item_is_a_leaf():
    t = oracle.tree_build(_rows([[(0, 100)]], 10))
    assert t["nodes"] == 1 and t["kind"][0] == 0 and t["count"][0] == 1


def test_under_threshold_is_a_leaf():
    t = oracle.tree_build(_rows([[(0, (i + 1) * 100)] for i in range(8)], 10), leaf_threshold=16)
    assert t["nodes"] == 1 and t["count"][0] == 8


def test_over_threshold_creates_a_branch():
    rows = _rows([[(0, (i - 10) * 1000 or 1)] for i in range(20)], 10)
    t = oracle.tree_build(rows, leaf_threshold=4)
    assert t["kind"][0] == 1


def test_preserves_all_elements_and_bounds_leaves():
    rows = _rows([[(i % 10, (i + 1) * 100)] for i in range(50)], 20)
    t = oracle.tree_build(rows, leaf_threshold=4)
    assert t["occupants"] == 50 and sorted(t["perm"]) == list(range(50))
    rows = _rows([[(0, (i % 10 + 1) * 100), (1, (i // 10 + 1) * 200)] for i in range(100)], 5)
    t = oracle.tree_build(rows, leaf_threshold=8)
    assert max(t["count"][t["kind"] == 0]) <= 16


def test_deterministic_and_split_dims_in_bounds():
    rows = _rows([[(i % 8, (i + 1) * 77)] for i in range(40)], 16)
    a, b = oracle.tree_build(rows, 4), oracle.tree_build(rows, 4)
    assert _shape(a)[0] == _shape(b)[0]
    rows = _rows([[(3, 100), (7, 200)], [(3, -100), (7, -200)], [(3, 500), (7, 300)], [(3, -500), (7, -300)]], 10)
    t = oracle.tree_build(rows, leaf_threshold=2)
    assert all(d < 10 for d in t["dim"][t["kind"] == 1])


def test_known_split_median_and_partition_order():
    """Hand-derived from EmbeddingLatticeBuilder: variance of dimension 3 (4 * 520000 - 0) beats
    dimension 7 (4 * 260000); sorted dimension-3 values [-500, -100, 100, 500] give the median
    values[2] = 100; the two-pointer partition swaps items 0 and 3, then stops with boundary 2."""
    rows = _rows([[(3, 100), (7, 200)], [(3, -100), (7, -200)], [(3, 500), (7, 300)], [(3, -500), (7, -300)]], 10)
    t = oracle.tree_build(rows, leaf_threshold=2)
    assert _shape(t)[0] == "B(3,100,L(2),L(2))"
    assert list(t["perm"]) == [3, 1, 2, 0]
    assert list(t["start"][1:]) == [0, 2]


def test_equal_values_stop_the_split():
    """All values of the widest dimension equal except one: the median equals the majority value,
    nothing is below it only when the odd value is larger, and a side left empty makes a leaf."""
    rows = _rows([[(0, 5)]] * 10 + [[(0, 9)]], 3)
    t = oracle.tree_build(rows, leaf_threshold=2)
    assert t["nodes"] == 1 and t["count"][0] == 11


def test_all_zero_rows_have_no_split_dimension():
    t = oracle.tree_build(np.zeros((40, 6), np.int64), leaf_threshold=4)
    assert t["nodes"] == 1 and t["count"][0] == 40


def _build_items(count):
    return _rows([[(0, ((i * 37) % 100 + 1) * 10), (1, ((i * 73) % 100 + 1) * 10)] for i in range(count)], 5)


def test_serializer_round_trip_and_identical_bytes():
    rows = _build_items(40)
    payload = np.arange(40, dtype=np.int32)
    a = oracle.slat_save(rows, payload, leaf_threshold=4)
    assert a == oracle.slat_save(rows, payload, leaf_threshold=4)
    loaded = oracle.slat_load(a)
    built = oracle.tree_build(rows, 4)
    for k in INFO:
        assert loaded[k] == built[k], k
    # occupants come back in leaf order with their payloads and components
    np.testing.assert_array_equal(loaded["payload"], built["perm"])
    np.testing.assert_array_equal(loaded["rows"], rows[built["perm"]])
    assert _shape(loaded)[0] == _shape(built)[0]


def test_serializer_record_layout():
    """Leaf record: tag, count, then per occupant TotalDimensions, entry count, (ushort, long)
    entries of the nonzero components in ascending dimension, Int32 payload."""
    rows = _rows([[(0, 12345), (3, -67890)]], 10)
    b = oracle.slat_save(rows, np.array([7], np.int32))
    expect = struct.pack("<IHBi", 0x544C4153, 1, 0, 1) + struct.pack("<ii", 10, 2) + \
        struct.pack("<Hq", 0, 12345) + struct.pack("<Hq", 3, -67890) + struct.pack("<i", 7)
    assert b == expect
    rows = _rows([[(3, 100), (7, 200)], [(3, -100), (7, -200)], [(3, 500), (7, 300)], [(3, -500), (7, -300)]], 10)
    b = oracle.slat_save(rows, np.arange(4, dtype=np.int32), leaf_threshold=2)
    assert b[6:18] == struct.pack("<BHqB", 1, 3, 100, 3)


@pytest.mark.parametrize("data,status", [
    (bytes([0x00, 0x01, 0x02, 0x03, 0x00, 0x01]), 2),                     # invalid magic
    (struct.pack("<IH", 0x544C4153, 99), 2),                              # invalid version
    (struct.pack("<IHB", 0x544C4153, 1, 7), 2),                           # unknown node tag
    (struct.pack("<IH", 0x544C4153, 1), 5),                               # no root node
    (struct.pack("<IHBi", 0x544C4153, 1, 0, 2) + struct.pack("<ii", 4, 0), 5),  # truncated leaf
    (struct.pack("<IHBi", 0x544C4153, 1, 0, 1) + struct.pack("<ii", 4, 1) + struct.pack("<Hq", 1, 0) +
     struct.pack("<i", 0), 1),                                            # zero-valued entry
    (struct.pack("<IHBi", 0x544C4153, 1, 0, 1) + struct.pack("<ii", 4, 2) + struct.pack("<Hq", 2, 5) +
     struct.pack("<Hq", 1, 5) + struct.pack("<i", 0), 1),                 # entries out of order
    (struct.pack("<IHBi", 0x544C4153, 1, 0, 1) + struct.pack("<ii", 0, 0) + struct.pack("<i", 0), 1),  # no dims
])
def test_serializer_load_errors(data, status):
    with pytest.raises(oracle.OracleError) as e:
        oracle.slat_load(data)
    assert e.value.status == status


def test_serializer_branch_without_children_loads():
    """A branch whose child mask is 0 is legal in the format (ReadBranch keeps null children)."""
    data = struct.pack("<IHBHqB", 0x544C4153, 1, 1, 2, 50, 0)
    t = oracle.slat_load(data)
    assert (t["nodes"], t["branches"], t["leaves"], t["occupants"]) == (1, 1, 0, 0)
