"""B200 (sm_100a) expert-parallel MoE layer behind the reference's entry points.

Modules (each loads ``_lib/libmoe_ep.so`` through ``_native``; there is no
CPU fallback):

* ``alltoall_persistent_gemm.run`` — the fused dispatch + grouped GEMM, padded
  (the reference's contract) or unpadded (``general_a2a=True``);
* ``baseline.run`` — the same output contract with the reference's NCCL
  baseline signature;
* ``utils`` — device routing (``route``, ``dispatch``, ``pack_padded``,
  ``pack_compact``), the router (``router``), ``gen_tensor``;
* ``combine`` — the layer with its return path and top-k combine;
* ``mlp`` — the full gated expert MLP behind the exchange;
* ``symm`` — the cuMem symmetric workspaces; ``workloads`` — seeded inputs;
* ``build`` — compiles the library in-tree.
"""
