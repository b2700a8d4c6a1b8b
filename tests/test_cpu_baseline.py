"""The C4 CPU baseline (oracle/cpu_baseline.py): a bounded sample timed on one
thread and on several, reported in the same algorithmic GB/s as the GPU line."""

from oracle import cpu_baseline


def test_paged_attention_cpu_baseline_reports_both_thread_counts():
    r = cpu_baseline.paged_attention_gbs(sequences=2, threads=2, seed=1)
    assert r["gbs_1_thread"] > 0 and r["gbs_all_threads"] > 0
    assert r["threads"] == 2 and "2 sequences" in r["sample"]
