"""Live 1P1D serving harness: exclusive-GPU gate, proxy, worker HTTP API,
paired benchmark client, fail-closed launcher, validity-gated aggregation,
input-trace verification and preregistered job queues."""
