"""Benchmark data and metrics: LongBench / LongBench-v2, RULER qa_2 packs, chunk priority schedules."""
