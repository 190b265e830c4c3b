"""The ncu raw-CSV summariser on a synthetic capture (no GPU, no ncu run):
units are honoured, thousands separators parsed, the three largest stall
reasons reported, and achieved rates derived from the duration."""
from sched_pass_b200.benchmarks import ncu_summary as S

CSV = '''"ID","Kernel Name","gpu__time_duration.sum","dram__bytes_read.sum","dram__bytes_write.sum","gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed","sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active","launch__registers_per_thread","smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio","smsp__average_warps_issue_stalled_wait_per_issue_active.ratio","smsp__average_warps_issue_stalled_barrier_per_issue_active.ratio","smsp__average_warps_issue_stalled_membar_per_issue_active.ratio"
"","","usecond","Mbyte","Kbyte","%","%","register/thread","ratio","ratio","ratio","ratio"
"0","gemm_kernel<16, 1>","48.6","237.1","5,300","61.0","3.5","136","4.2","1.1","0.3","2.0"
"1","add_rmsnorm_kernel<256, 2>","10","20","0","40","0","40","0","0","0","0"
'''


def test_parse_and_summarize():
    rows = S.parse(CSV)
    assert [r["kernel"] for r in rows] == ["gemm_kernel<16, 1>", "add_rmsnorm_kernel<256, 2>"]
    peaks = {"hbm_gbs": 6500.0, "bf16_tflops": 1500.0}
    s = S.summarize(rows[0], peaks, alg_flops=2 * 16 * 28672 * 4096)
    assert abs(s["us"] - 48.6) < 1e-9
    assert abs(s["dram_MB"] - (237.1 + 5.3)) < 1e-6
    assert abs(s["dram_GBps"] - 242.4e6 / 48.6e-6 / 1e9) < 1e-6
    assert s["stalls"] == ["long_scoreboard", "membar", "wait"]
    assert s["regs"] == 136 and s["tensor_pct"] == 3.5
    assert abs(s["alg_TFLOPs"] - 2 * 16 * 28672 * 4096 / 48.6e-6 / 1e12) < 1e-9
    md = S.markdown([s, S.summarize(rows[1], peaks)])
    assert md.count("\n") == 3 and "gemm_kernel<16, 1>" in md and "long_scoreboard" in md
