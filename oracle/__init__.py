"""CPU oracle for the streaming FastConformer step, its per-stream caches and the RNN-T greedy step.

TEST INFRASTRUCTURE ONLY. Nothing in the product (the CUDA library and its host bindings) imports,
links or runs this package. Only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline legs of
`bench.py` use it, and there only as the checker or as the timed CPU baseline.

Modules:
  weights     seeded random weights under the NeMo checkpoint tensor names
  stream_step restatement of the cache-aware streaming encoder step (subsampling, 24 macaron layers with
              rel-pos attention and causal conv, joint encoder projection)
  rnnt        restatement of the RNN-T prediction net, joint and greedy decoding with carried state
  cache_ring  bit-exact model of the paged per-stream ring caches (append / roll / gather / evict)

Parity is pinned against the reference's own Python code (`tools/nemotron_ane.py`,
`reference/nemo/check_spec.py`) through the fixtures in `tests/golden/`, which
`tests/golden/make_golden.py` generates by importing those files unchanged.
"""
