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
