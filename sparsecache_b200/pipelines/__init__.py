"""Experiment pipelines: CacheBlend reuse (one-shot and progressive) and P/D progressive runs."""
