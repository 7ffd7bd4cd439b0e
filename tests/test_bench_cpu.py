"""CPU checks of the bench's roofline arithmetic and its launch-list summary (no GPU needed)."""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test",
                                                  os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_flop_per_pbs_matches_the_roofline_formula(bench):
    # n [((k+1) l + (k+1)) 5 (N/2) log2(N/2) + (k+1)^2 l (N/2) 8], the FFT-equivalent count
    assert bench.flop_per_pbs() == 834 * (4 * 51200 + 32768) == bench.FLOP_PER_PBS
    assert bench.flop_per_pbs(levels=2) == 834 * (6 * 51200 + 2 * 32768)
    assert bench.flop_per_pbs(n=1024, N=8192) == 1024 * (4 * 5 * 4096 * 12 + 4 * 4096 * 8)
    # every extra gadget level adds two forward transforms and two products per CMux
    step = bench.flop_per_pbs(levels=3) - bench.flop_per_pbs(levels=2)
    assert step == 834 * (2 * 51200 + 4 * 1024 * 8)


def test_summarize_launches_aggregates_per_kernel(bench, tmp_path, capsys):
    csv = tmp_path / "launches.csv"
    csv.write_text(
        '==PROF== Connected to process 1\n'
        '"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream",'
        '"Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit",'
        '"Metric Value"\n'
        '"0","1","python","h","void pnb::blind_rotate_tm_kernel<4>(const unsigned long *)","1",'
        '"7","(256, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics",'
        '"gpu__time_duration.sum","ms","6.50"\n'
        '"1","1","python","h","pnb::ks_gemm_kernel(int)","1","7","(192, 1, 1)","(108, 1, 1)",'
        '"0","10.0","Command line profiler metrics","gpu__time_duration.sum","us","250.00"\n'
        '"2","1","python","h","void pnb::blind_rotate_tm_kernel<4>(const unsigned long *)","1",'
        '"7","(256, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics",'
        '"gpu__time_duration.sum","ms","6.25"\n')
    bench.summarize_launches(str(csv))
    out = capsys.readouterr().out.splitlines()
    assert len(out) == 4  # header, one line per kernel, the total
    rot = next(line for line in out if "blind_rotate_tm_kernel" in line).split()
    ks = next(line for line in out if "ks_gemm_kernel" in line).split()
    assert rot[-3:] == ["2", "12.75", "98.08%"]
    assert ks[-3:] == ["1", "0.25", "1.92%"]
    assert out[-1].split()[-2:] == ["3", "13.00"]
