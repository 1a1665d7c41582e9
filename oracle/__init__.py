"""CPU oracle for the StageML MoE-LoRA residual path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's algorithm for this path, used by
``tests/`` as the checker of the CUDA kernels, by ``__graft_entry__.smoke()``
and by ``bench.py``'s CPU baseline. Nothing in the product (``stageml_b200``)
imports it: the product path runs the sm_100a kernels or fails.

Every function cites the reference file:line it restates. The restatement is
pinned against golden vectors produced by running the reference itself
(``tests/golden/make_golden.py``; checked by ``tests/test_oracle_golden.py``):
the MoE-LoRA layers, the adapter bank and cost-based cache, the LoRA fold,
``_fallback_moe``, the SwiGLU ``RequestExecutor`` and the router
``make_routing``. Where the reference has no code (LoRA on w3/w2, shared
experts, FP8 weights, the explicit permutation) the oracle states the
convention used and says so in the function's docstring.
"""
