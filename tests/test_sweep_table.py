"""The sweep's table builder (host logic only) and the committed table's coverage."""

from muse_bf16_proj_b200 import _lib
from muse_bf16_proj_b200.dispatch import Dispatch
from muse_bf16_proj_b200.sweep import table_entries


def R(fmt, plan, us):
    return {"fmt": fmt, "plan": plan, "us": us}


def test_table_entries_ranges_and_12b_rows():
    rows = [
        {"n": 10, "k": 512, "m": 1, "best": R("12b", {"kernel": "gemv_12b"}, 5), "best_bf16": R("bf16", {"kernel": "gemv_bf16"}, 6)},
        {"n": 10, "k": 512, "m": 2, "best": R("12b", {"kernel": "gemv_12b"}, 5), "best_bf16": R("bf16", {"kernel": "tc_tile", "split": 2}, 6)},
        {"n": 10, "k": 512, "m": 4, "best": R("bf16", {"kernel": "tc_tile", "split": 2}, 5), "best_bf16": R("bf16", {"kernel": "tc_tile", "split": 2}, 5)},
        {"n": 10, "k": 512, "m": 8, "best": R("bf16", {"kernel": "tc_tile", "split": 3}, 5), "best_bf16": R("bf16", {"kernel": "tc_tile", "split": 3}, 5)},
        {"n": 10, "k": 512, "m": 16, "best": None, "best_bf16": None},
    ]
    e = table_entries(rows)
    assert [(x["m_lo"], x["m_hi"], x["weights"], x["plan"]["kernel"]) for x in e] == [
        (1, 2, "12b", "gemv_12b"), (1, 1, "bf16", "gemv_bf16"), (2, 4, "bf16", "tc_tile"), (5, 8, "bf16", "tc_tile")]
    d = Dispatch(entries=e)
    assert d.plan(2, 10, 512, have_12b=True)[1] == "12b"
    plan, fmt = d.plan(2, 10, 512, have_12b=False)
    assert fmt == "bf16" and plan.split == 2
    assert d.plan(6, 10, 512)[0].split == 3
    assert d.plan(12, 10, 512)[0].kernel in _lib.KERNEL_NAMES  # past the table: library default


def test_committed_table_covers_reference_shapes_when_present():
    d = Dispatch()
    if not d.entries:
        return
    shapes = {(e["n"], e["k"]) for e in d.entries}
    for n, k in ((2304, 8192), (8192, 1024), (4096, 8192), (8192, 4096), (1024, 4096), (6144, 4096)):
        assert (n, k) in shapes, (n, k)
        for m in (1, 16, 256):
            if (n, k) == (1024, 4096) and m > 8:
                continue
            plan, _ = d.plan(m, n, k)
            assert plan.kernel in _lib.KERNEL_NAMES


def test_merge_replaces_only_the_swept_shapes():
    from muse_bf16_proj_b200.sweep import merge_entries
    old = [{"n": 10, "k": 512, "m_lo": 1, "m_hi": 4, "weights": "bf16", "plan": {"kernel": "tc_tile"}},
           {"n": 20, "k": 512, "m_lo": 1, "m_hi": 4, "weights": "bf16", "plan": {"kernel": "tc_tile"}},
           {"n": 20, "k": 512, "m_lo": 1, "m_hi": 2, "weights": "12b", "plan": {"kernel": "gemv_12b"}}]
    new = [{"n": 20, "k": 512, "m_lo": 1, "m_hi": 8, "weights": "12b", "plan": {"kernel": "gemv_12t"}}]
    got = merge_entries(old, new)
    assert [(e["n"], e["weights"], e["plan"]["kernel"]) for e in got] == [(10, "bf16", "tc_tile"), (20, "12b", "gemv_12t")]


def test_merge_of_a_small_m_sweep_keeps_larger_m_and_faster_12b_rows():
    from muse_bf16_proj_b200.sweep import merge_entries
    old = [{"n": 20, "k": 512, "m_lo": 1, "m_hi": 2, "weights": "12b", "plan": {"kernel": "gemv_12t"}, "us": {"1": 5.0, "2": 6.0}},
           {"n": 20, "k": 512, "m_lo": 3, "m_hi": 4, "weights": "12b", "plan": {"kernel": "gemv_12b"}, "us": {"4": 9.0}},
           {"n": 20, "k": 512, "m_lo": 1, "m_hi": 8, "weights": "bf16", "plan": {"kernel": "tc_tile"},
            "us": {"1": 8.0, "2": 8.0, "4": 8.0, "8": 9.0}, "cublas_us": {"1": 10.0, "8": 11.0}},
           {"n": 20, "k": 512, "m_lo": 9, "m_hi": 16, "weights": "bf16", "plan": {"kernel": "tc_tile", "split": 2},
            "us": {"16": 10.0}}]
    new = [{"n": 20, "k": 512, "m_lo": 1, "m_hi": 4, "weights": "bf16", "plan": {"kernel": "gemv_tiles"},
            "us": {"1": 5.5, "2": 6.5, "4": 7.0}}]
    got = merge_entries(old, new, bf16_only=True)
    rows = [(e["weights"], e["m_lo"], e["m_hi"], e["plan"]["kernel"]) for e in got]
    # The 12-bit row faster at M = 1, 2 stays; the one slower at M = 4 goes; the old BF16 row is cut
    # to start above the swept range, keeping only its timings there; M > 8 is untouched.
    assert rows == [("12b", 1, 2, "gemv_12t"), ("bf16", 1, 4, "gemv_tiles"), ("bf16", 5, 8, "tc_tile"),
                    ("bf16", 9, 16, "tc_tile")]
    cut = got[2]
    assert cut["us"] == {"8": 9.0} and cut["cublas_us"] == {"8": 11.0}
    assert old[2]["m_lo"] == 1  # the committed rows are not modified in place
    d = Dispatch(entries=got)
    assert d.plan(1, 20, 512, have_12b=True)[1] == "12b"
    assert d.plan(3, 20, 512, have_12b=True)[0].kernel == _lib.KERNEL_GEMV_TILES
    assert d.plan(6, 20, 512)[0].kernel == _lib.KERNEL_TC_TILE
