"""Drop-in for edge35b/cpu_route.py cpu_forward (:23-80).

The reference computes the routed experts of one token on the host's AVX2
cores (cpu_experts.c) from the CPU expert banks, optionally sending reused
rows to the GPU ("hybrid").  On B200 the host-resident banks are instead
streamed over the host link into HBM slots inside the layer's device chain
(the "b200-host" / "b200-packed" residencies of ExpertPool), so both variants
run that chain; the shape checks and the result (eager ascending-expert BF16
adds) are the reference's.
"""

from __future__ import annotations

from lightreason_b200.fused_experts import check_single_token


def cpu_forward(layer, hidden, indices, weights, *, hybrid=False):
    check_single_token(layer, hidden, indices, weights,
                       "The AVX2 kernel requires the original 35B single-token expert layout")
    return layer.run(hidden, indices, weights)
