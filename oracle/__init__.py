"""Oracle: a CPU (numpy) restatement of the reference's routing and expert-
parallel layer, used only as the checker.

Test infrastructure.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` import this package; the library
(``nvshmem_testing_b200``) never does, and never falls back to it.

Pinning: ``tests/golden/`` holds fixtures produced by running the
reference's own code in a container where it is importable
(``tests/golden/make_golden.py``): ``utils.gen_tensor`` on CPU for routing
and padding, and ``baseline.run`` under gloo with two ranks for the layer
output.  ``tests/test_oracle.py`` checks this oracle against them.
"""
from .routing import bucketize, local_max, pad_coalesce, gen_tensor_restated, recv_counts_matrix  # noqa: F401
from .routing import compact_coalesce, uncompact_padded  # noqa: F401
from .layer import alltoall_equal, baseline_run, ep_layer, bf16_bits_to_f32, f32_to_bf16_bits, expert_cell  # noqa: F401
from .layer import route_slots, combine_layer, combine_from_outputs, compact_layer, compact_from_padded  # noqa: F401
from .layer import router, softmax_topk, topk_mismatches  # noqa: F401
from .layer import mlp_compact  # noqa: F401
