"""Benchmark harness: EP benchmark with an exact reference (`ep_benchmark`), routing tables with
controlled traffic (`routing`), result summaries (`summarize`)."""
