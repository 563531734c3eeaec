"""CPU: the ncu launch-list summariser on a synthetic ``--csv`` log."""
import pytest

from fack_b200 import ncu_launches as nl

HEADER = ('"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size",'
          '"Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"')


def row(i, kernel, unit, value, metric="gpu__time_duration.sum"):
    return (f'"{i}","1","python","box","{kernel}","1","7","(384, 1, 1)","(12, 2, 5)","0","10.0",'
            f'"Command line profiler metrics","{metric}","{unit}","{value}"')


GEMM = "void fack::gemm_bs_kernel<256, false>(CUtensorMap_st, CUtensorMap_st, fack::Params)"
RANDN = ("void at::native::(anonymous namespace)::distribution_elementwise_grid_stride_kernel<float, 4, "
         "at::native::templates::cuda::normal_and_transform<float, float>(at::TensorIteratorBase &)>(long, "
         "at::PhiloxCudaState, T3, T4)")

LOG = "\n".join([
    "==PROF== Connected to process 1234",
    "==PROF== Profiling \"gemm_bs_kernel\": 0%....50%....100% - 1 pass",
    HEADER,
    row(0, RANDN, "usecond", "10.50"),
    row(1, GEMM, "usecond", "17.25"),
    row(2, GEMM, "nsecond", "17,750"),
    row(3, GEMM, "usecond", "17.50"),
    row(3, GEMM, "byte", "123", metric="dram__bytes_read.sum"),      # other metrics are ignored
    "==PROF== Disconnected from process 1234",
])


def test_names_units_and_shares():
    launches = nl.read_launches(LOG)
    assert len(launches) == 4
    rows = nl.summarize(launches)
    assert [r[0] for r in rows] == ["fack::gemm_bs_kernel<256, false>",
                                    "at::native::distribution_elementwise_grid_stride_kernel<float, 4, "
                                    "at::native::templates::cuda::normal_and_transform<float, float>"
                                    "(at::TensorIteratorBase &)>"]
    k, n, total, per, share = rows[0]
    assert n == 3 and total == pytest.approx(52.5) and per == pytest.approx(17.5)
    assert share == pytest.approx(52.5 / 63.0)
    assert sum(r[4] for r in rows) == pytest.approx(1.0)
    table = nl.markdown(rows)
    assert "| `fack::gemm_bs_kernel<256, false>` | 3 | 52.5 | 17.50 | 83.3 % |" in table


def test_top_groups_the_rest():
    rows = nl.summarize(nl.read_launches(LOG), top=1)
    assert rows[-1][0] == "other (1 kernels)" and rows[-1][1] == 1 and rows[-1][2] == pytest.approx(10.5)


def test_bad_logs_refused():
    with pytest.raises(ValueError, match="header"):
        nl.read_launches("==PROF== nothing captured\n")
    with pytest.raises(ValueError, match="unknown time unit"):
        nl.read_launches(HEADER + "\n" + row(0, GEMM, "cycle", "5"))
    with pytest.raises(ValueError, match="no gpu__time_duration.sum rows"):
        nl.read_launches(HEADER + "\n" + row(0, GEMM, "byte", "5", metric="dram__bytes_read.sum"))
