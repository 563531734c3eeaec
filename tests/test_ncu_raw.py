"""CPU: the ncu raw-page reader on a synthetic ``--page raw --csv`` export."""
import pytest

from fack_b200 import ncu_raw

GEMM = "void fack::gemm_bs_kernel<256, false>(CUtensorMap_st, CUtensorMap_st, fack::Params)"
HEAD = ('"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size",'
        '"Device","CC","dram__bytes_read.sum","dram__bytes_write.sum","gpu__time_duration.sum",'
        '"launch__registers_per_thread","sm__throughput.avg.pct_of_peak_sustained_elapsed"')
UNITS = '"","","","","","","","","","","","Mbyte","Kbyte","usecond","register/thread","%"'


def launch(i, read, write, us, kernel=GEMM):
    return (f'"{i}","77","python","box","{kernel}","1","7","(384, 1, 1)","(12, 2, 5)","0","10.0",'
            f'"{read}","{write}","{us}","168","41.5"')


RAW = "\n".join(["==PROF== Disconnected", HEAD, UNITS,
                 launch(0, "23.96", "0", "17.45"), launch(1, "23.98", "12.5", "17.30"),
                 launch(2, "1.20", "0", "3.1", kernel="void at::native::vectorized_elementwise_kernel<4>(int)")])


def test_units_and_fields():
    recs = ncu_raw.read_raw(RAW)
    assert len(recs) == 3
    r = recs[1]
    assert r["kernel"] == "fack::gemm_bs_kernel<256, false>"
    assert r["dram_read"] == pytest.approx(23.98e6) and r["dram_write"] == pytest.approx(12.5e3)
    assert r["dram_bytes"] == pytest.approx(23.98e6 + 12.5e3)
    assert r["duration_us"] == pytest.approx(17.30) and r["registers"] == 168 and r["sm_pct"] == 41.5
    assert r["tensor_pct"] is None and r["dram_pct"] is None           # not in this capture
    assert "| 1 | `fack::gemm_bs_kernel<256, false>` | 17.30 | 23.99 |" in ncu_raw.markdown(recs)


def test_traffic_entry_for_selected_launches():
    recs = [r for r in ncu_raw.read_raw(RAW) if "gemm_bs" in r["kernel"]]
    e = ncu_raw.traffic_entry(recs, "decode", "ncu raw page prof.csv")
    assert e["decode"]["bytes_per_launch"] == round((23.96e6 + 23.98e6 + 12.5e3) / 2)
    assert e["decode"]["kernel"] == "fack::gemm_bs_kernel<256, false>"


def test_bad_exports_refused():
    with pytest.raises(ValueError, match="header"):
        ncu_raw.read_raw("nothing here\n")
    with pytest.raises(ValueError, match="unknown unit"):
        ncu_raw.read_raw("\n".join([HEAD, UNITS.replace('"Mbyte"', '"Mibyte"'), launch(0, "1", "0", "1")]))
    with pytest.raises(ValueError, match="no dram"):
        ncu_raw.traffic_entry([{"dram_bytes": None, "kernel": "k"}], "x", "s")
