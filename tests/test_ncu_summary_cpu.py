"""ncu_summary.py on a raw-page CSV (the text `ncu --import R --page raw --csv`
prints), without a GPU: the launch picked, units scaled, the derived roofline
rows and the traffic file bench.py reads."""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "aegis-core_b200", "tune"))
import ncu_summary as ns  # noqa: E402

CSV = (
    '"ID","Kernel Name","gpu__time_duration.sum","dram__bytes_read.sum","dram__bytes_write.sum",'
    '"sm__ops_path_tensor_op_utchmma_src_bf16_dst_fp32_sparsity_off.avg.pct_of_peak_sustained_elapsed",'
    '"launch__grid_size"\n'
    '"","","us","Mbyte","Mbyte","%",""\n'
    '"0","splitk_reduce_kernel","5.0","10.0","2.0","0",""\n'
    '"1","umma2_gemm_kernel<bf16>","700.0","876.5","125.2","88.47","2048"\n'
    '"2","nvjet_tst_256x256","650.0","856.0","125.0","93.2","148"\n'
)


def test_summary_table_picks_the_launch_and_derives_the_roofline(tmp_path):
    p = tmp_path / "umma2.csv"
    p.write_text(CSV)
    out_json = tmp_path / "t.json"
    import io
    import contextlib
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        ns.main(["--csv", str(p), "--kernel", "umma2", "--flops", str(2.0 * 8192 ** 3), "--bytes",
                 str(3 * 2 * 8192 ** 2), "--peak-tflops", "1651.8", "--traffic-json", str(out_json),
                 "--command", "python bench.py ..."])
    text = buf.getvalue()
    assert "umma2_gemm_kernel<bf16>" in text and "88.47 %" in text and "2048" in text
    assert "| traffic (DRAM read + write per launch) | 1001.70 MB |" in text
    assert "| achieved TFLOP/s (algorithmic flops / duration) | 1570.7 |" in text  # 1.0995e12 / 700 us
    assert "| fraction of the TFLOP/s peak | 0.951 |" in text
    t = json.loads(out_json.read_text())
    assert t["dram_bytes_per_launch"] == 876.5e6 + 125.2e6 and t["command"] == "python bench.py ..."


def test_default_is_the_last_launch(tmp_path):
    p = tmp_path / "r.csv"
    p.write_text(CSV)
    m = ns.parse(p.read_text())
    assert m["Kernel Name"][0] == "nvjet_tst_256x256"
    assert ns.number(m, "gpu__time_duration.sum") == 650e-6
