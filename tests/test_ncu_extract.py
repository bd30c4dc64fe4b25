"""ncu export parsing (no GPU): kernel-name shortening, both CSV layouts,
unit normalisation, and rejection of a file without metrics. Mirrors the
contract of the reference's tests/test_ncu_extract.py for our kernels."""

import pytest

from flashattn_cuda import ncu_extract


@pytest.mark.parametrize(
    "mangled,expected",
    [
        ("void fa::prefill::prefill_kernel(CUtensorMap_st, CUtensorMap_st, __half *, int)",
         "prefill_kernel"),
        ("fa::decode::decode_kernel(fa::DecodeArgs)", "decode_kernel"),
        ("void (anonymous namespace)::prefill_kernel<(bool)1>(const __half *, int)",
         "prefill_kernel<(bool)1>"),
        ("void (anonymous namespace)::prefill_kernel<(bool)0>(const __half *, int)",
         "prefill_kernel<(bool)0>"),
        ("void at::native::foo<int, (bool)1>(x)", "foo<int, (bool)1>"),
        ("simple_kernel", "simple_kernel"),
    ],
)
def test_short_kernel_name(mangled, expected):
    assert ncu_extract.short_kernel_name(mangled) == expected


LONG_CSV = '''==PROF== Connected to process 1
"ID","Process ID","Kernel Name","Section Name","Metric Name","Metric Unit","Metric Value"
"0","1","fa::decode::decode_kernel(fa::DecodeArgs)","Memory","dram__bytes_read.sum.per_second","Tbyte/second","5.573"
"0","1","fa::decode::decode_kernel(fa::DecodeArgs)","Memory","dram__bytes_read.sum","Mbyte","808.4"
"0","1","fa::decode::decode_kernel(fa::DecodeArgs)","Occupancy","sm__warps_active.avg.pct_of_peak_sustained_active","%","27.9"
"0","1","fa::decode::decode_kernel(fa::DecodeArgs)","SOL","gpu__time_duration.sum","usecond","145.056"
'''

WIDE_CSV = '''"ID","Kernel Name","gpu__time_duration.sum","sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active"
"","","usecond","%"
"0","void fa::prefill::prefill_kernel(CUtensorMap_st, int)","171.136","34.4"
'''


def test_parse_long_format_and_render(tmp_path):
    p = tmp_path / "d.csv"
    p.write_text(LONG_CSV)
    parsed = ncu_extract.parse(str(p))
    table = ncu_extract.kernel_table(parsed)
    assert "`decode_kernel`" in table
    assert "5573.0 GB/s" in table          # Tbyte/s normalised to GB/s
    assert "808,400,000 B" in table        # Mbyte normalised to bytes
    assert "145,056 ns" in table           # us normalised to ns
    assert "27.9%" in table
    assert "Tensor pipe active" not in table  # absent metrics are dropped


def test_parse_wide_raw_page(tmp_path):
    p = tmp_path / "p.csv"
    p.write_text(WIDE_CSV)
    table = ncu_extract.kernel_table(ncu_extract.parse(str(p)))
    assert "`prefill_kernel`" in table
    assert "34.4%" in table and "171,136 ns" in table


def test_parse_rejects_a_csv_without_metrics(tmp_path):
    bad = tmp_path / "bad.csv"
    bad.write_text('"a","b"\n"1","2"\n')
    with pytest.raises(SystemExit):
        ncu_extract.parse(str(bad))
