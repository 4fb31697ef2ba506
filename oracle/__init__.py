"""CPU oracle for the weight-quantised matmul hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference's own arithmetic for every function on the path
(each function cites the reference file:line it follows). It is the checker: only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline legs may import it. The product path
(mq/) never imports it and has no CPU fallback.

Parity pinning: the reference ships no golden tensors. The restatements are pinned against
(a) the reference's own Python run here (llama/run.py quantize4, qwen3moe/reference.py
Weights.int4, lfm2/weights.py dequant_q4_0), whose outputs are committed as fixtures under
tests/golden/ by tests/golden/make_golden.py, and (b) the reference's C/C++ converters compiled
from their sources under oracle/_ref/ by oracle/Makefile. The reference's Mojo kernels cannot
run here (no Mojo, no Vulkan); the matmul sums they compute are restated directly.
"""
