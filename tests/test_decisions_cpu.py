"""Decision-log reader and counterfactual pricing (ferry_b200.decisions) on a
log written here byte for byte in the executor's format; truncated and foreign
files are rejected."""
import struct

import pytest

from ferry_b200 import decisions


def _write(path, hdr, recs):
    with open(path, "wb") as f:
        f.write(struct.pack("<4sI14i", b"FRYD", 1, *[hdr[k] for k in decisions.FIELDS]))
        for r, tasks in recs:
            f.write(struct.pack("<qiiqqqiidffq", *r))
            for t in tasks:
                f.write(struct.pack("<iiiiq", *t))


HDR = dict(rank=1, world=2, num_requests=8, num_layers=2, kv_heads=4, max_pages=64, cache_pages=16, top_k=8,
           unit_bytes=8192, steps_per_req=10, migrate_mode=1, steal_batch=4, max_batch=4, cost_filter=0)


def test_read_and_price(tmp_path):
    p = tmp_path / "r1.log"
    recs = [((3, 0, 0, 5, 1, 9, 2, 2, 2.0, 0.05, 0.0, 40 * 8192), [(7, 4, 3, 0, 25), (2, 9, 1, 1, 15)]),
            ((8, 0, 1, 2, 0, 4, 1, 1, 2.5, 0.01, 0.0, 0), [(5, 0, 2, 2, 0)])]
    _write(p, HDR, recs)
    hdr, ds = decisions.read_log(str(p))
    assert hdr == HDR and len(ds) == 2
    d0 = ds[0]
    assert (d0.tick, d0.victim, d0.fair, d0.own_occupancy, d0.victim_size, d0.planned, d0.taken) == (3, 0, 5, 1, 9, 2, 2)
    assert d0.tasks[0].request == 7 and d0.tasks[0].resident_units == 25 and ds[1].forced
    rows = decisions.price(hdr, d0, nvlink_gbs=800.0, host_gbs=50.0, fixed_ms=0.06)
    by = {(r[0], r[1]): r for r in rows}
    # request 7 at step 4: 6 steps left at 2 ms; 25 resident units of 8 KiB
    assert by[("a0", 7)][4] == pytest.approx(12.0)
    assert by[("delta", 7)][2] == 25 * 8192
    assert by[("delta", 7)][4] == pytest.approx(25 * 8192 / 800e6 + 0.06)
    assert by[("full", 7)][2] == 2 * 4 * 16 * 8192
    assert by[("drop", 7)][3] == 25 * 8192 and by[("drop", 7)][2] == 0
    assert by[("delta", 7)][2] + by[("delta", 2)][2] == d0.mig_bytes  # delta moved exactly the resident pages
    csv = decisions.counterfactuals([str(p)], 800.0, 50.0)
    assert csv[0][0] == "decision" and len(csv) == 1 + 4 * 3
    cheapest = [r for r in csv[1:] if r[8] == 5 and r[14] == 1]
    assert len(cheapest) >= 1 and cheapest[0][9] in ("delta", "drop")  # nothing resident: free to move


def test_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.log"
    p.write_bytes(b"NOPE" + bytes(60))
    with pytest.raises(ValueError):
        decisions.read_log(str(p))
    q = tmp_path / "trunc.log"
    _write(q, HDR, [((3, 0, 0, 5, 1, 9, 2, 2, 2.0, 0.05, 0.0, 0), [(7, 4, 3, 0, 25)])])
    q.write_bytes(q.read_bytes()[:-10])
    with pytest.raises(ValueError):
        decisions.read_log(str(q))
