"""CPU: the launch-list summariser behind the tables in profiles/
(malus_b200/profsum.py) on a synthetic ncu CSV in ncu's own format: one row
per launch and metric, kernel names with template arguments, argument lists
and anonymous namespaces, mixed time and byte units."""
import csv
import io

import pytest

from malus_b200 import profsum

HEADER = ["ID", "Process ID", "Process Name", "Host Name", "Kernel Name", "Context", "Stream", "Block Size",
          "Grid Size", "Device", "CC", "Section Name", "Metric Name", "Metric Unit", "Metric Value"]


def _csv(tmp_path, rows):
    buf = io.StringIO()
    w = csv.writer(buf, quoting=csv.QUOTE_ALL)
    w.writerow(HEADER)
    for name, metric, unit, value, launch_id in rows:
        w.writerow([str(launch_id), "1", "python", "h", name, "1", "7", "(256, 1, 1)",
                    "(148, 1, 1)", "0", "10.0", "Command line profiler metrics", metric, unit, value])
    p = tmp_path / "launches.csv"
    # ncu writes a few "==PROF==" lines before the table; they must be skipped
    p.write_text("==PROF== Connected to process 1\n" + buf.getvalue())
    return p


def launch(i, name, ns=None, nbytes=None):
    out = []
    if ns is not None:
        out.append((name, "gpu__time_duration.sum", "nsecond", f"{ns:,}", i))
    if nbytes is not None:
        out.append((name, "dram__bytes_read.sum", "Mbyte", str(nbytes / 2e6), i))
        out.append((name, "dram__bytes_write.sum", "Mbyte", str(nbytes / 2e6), i))
    return out


def test_short_names():
    assert profsum.short_name("void malus::(anonymous namespace)::k_gemm_tc<0, 192, 16, true>(CUtensorMap, int)") \
        == "k_gemm_tc<0, 192, 16, true>"
    assert profsum.short_name("malus::<unnamed>::k_embed2(const int *, float *)") == "k_embed2"
    assert profsum.short_name("void k_splitk_reduce<0>(malus::TcKernelParams)") == "k_splitk_reduce<0>"


def test_durations_window_and_shares(tmp_path):
    rows = []
    i = 0
    for step in range(3):                      # three steps, each starting at k_embed2
        for name, ns in (("k_embed2(int*)", 1000), ("k_gemm_tc<0, 192, 16, 1>(int)", 6000),
                         ("k_gemm_tc<0, 192, 16, 1>(int)", 2000), ("k_colsum(float*)", 1000)):
            rows += launch(i, "void malus::(anonymous namespace)::" + name, ns=ns)
            i += 1
    ls = profsum.read_launches(_csv(tmp_path, rows))
    assert len(ls) == 12 and all(d["bytes"] is None for d in ls)
    win = profsum.window(ls, "k_embed2", 2)
    assert len(win) == 8                       # the last two steps
    table, tot = profsum.summarise(win, 6546.0)
    assert tot["launches"] == 8 and tot["ms"] == pytest.approx(0.020)
    top = table[0]
    assert top["kernel"] == "k_gemm_tc<0, 192, 16, 1>" and top["launches"] == 4
    assert top["ms"] == pytest.approx(0.016) and top["share"] == pytest.approx(0.8)
    md = profsum.markdown(table, tot)
    assert md.splitlines()[0] == "launches 8, summed device time 0.020 ms"
    assert "| k_gemm_tc<0, 192, 16, 1> | 4 | 0.016 | 80.0% |" in md


def test_dram_columns(tmp_path):
    rows = launch(0, "void k_gemm_tc<1, 192, 16, false>(int)", ns=100_000, nbytes=250e6)
    rows += launch(1, "void k_gemm_tc<1, 192, 16, false>(int)", ns=100_000, nbytes=250e6)
    table, tot = profsum.summarise(profsum.read_launches(_csv(tmp_path, rows)), 5000.0)
    r = table[0]
    assert r["mb_per_launch"] == pytest.approx(250.0)
    assert r["gbs"] == pytest.approx(2500.0) and r["of_hbm"] == pytest.approx(0.5)
    assert "| 250.0 | 2500 | 0.50 |" in profsum.markdown(table, tot)


def test_window_without_enough_markers_keeps_everything(tmp_path):
    rows = launch(0, "void k_a(int)", ns=10) + launch(1, "void k_b(int)", ns=10)
    ls = profsum.read_launches(_csv(tmp_path, rows))
    assert profsum.window(ls, "k_embed2", 2) == ls
    assert profsum.window(ls, None, 2) == ls
