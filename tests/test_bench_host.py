"""CPU: bench.py's host-side pieces -- the DRAM-traffic figure taken from an ncu launch-list CSV
(one step's conv launches only, units scaled), the seeded per-image inputs the output check
regenerates, and the sampled rows of each shard."""
import sys

import numpy as np

from conftest import ROOT

sys.path.insert(0, str(ROOT))
import bench  # noqa: E402

HEAD = '"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size",' \
       '"Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"\n'


def row(i, kernel, metric, unit, value):
    return f'"{i}","1","p","h","{kernel}","1","13","(1,1,1)","(1,1,1)","0","10.0","s","{metric}","{unit}","{value}"\n'


def test_traffic_from_ncu_csv(tmp_path):
    p = tmp_path / "l.csv"
    p.write_text("==PROF== noise\n" + HEAD +
                 row(0, "void unnamed>::conv_tc_kernel<0, 4, 16>(P)", "dram__bytes_read.sum", "Mbyte", "2") +
                 row(0, "void unnamed>::conv_tc_kernel<0, 4, 16>(P)", "dram__bytes_write.sum", "byte", "1,000") +
                 row(1, "void unnamed>::dw_kernel<3, 1, 0, 7>(P)", "dram__bytes_read.sum", "byte", "5000") +
                 row(2, "void unnamed>::conv_rows_kernel<0, 4>(P)", "dram__bytes_read.sum", "byte", "3000") +
                 row(3, "void unnamed>::conv_rows_kernel<0, 4>(P)", "dram__bytes_read.sum", "byte", "999999"))
    got = bench.traffic_from_ncu_csv(p, images=2, step_launches=3)
    assert got["conv_dram_bytes_per_image"] == (2_000_000 + 1000 + 3000) // 2
    assert got["conv_launches"] == 2


def test_seeded_inputs_and_samples():
    a = bench.image_input(17, 300)
    assert a.dtype == np.int8 and a.size == 300
    np.testing.assert_array_equal(a, bench.image_input(17, 300))
    assert not np.array_equal(a, bench.image_input(18, 300))
    assert bench.sample_rows(512) == [0, 256, 511]
    assert bench.sample_rows(1) == [0]
