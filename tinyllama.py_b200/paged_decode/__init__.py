"""Host-side pieces around the cscr ops: layer glue, device-side decode
metadata, length-balanced sharding across GPUs and the seeded workloads the
tests and the benchmark share."""
