"""CPU oracle for the capped-KV decode path -- TEST INFRASTRUCTURE ONLY.

This package is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import it.  The CUDA product path in
``kvcacheboundaryprotection_b200`` never imports, calls or falls back to anything here.

What it restates (all citations are paths inside the reference project,
Gpgabriel25/KVCacheBoundaryProtection):

* ``oracle.policies``  -- the victim-selection policies and the structural
  prefix/suffix protection wrapper
  (``src/counterfact_kv_eviction/policies.py:12-63,181-196,1190-1449``,
  ``scripts/run_v3_jax.py:102-136``).
* ``oracle.generator`` -- the global-mask decode/eviction loop
  (``src/counterfact_kv_eviction/kv_coupled_generator.py:135-604``) plus the
  slot-layout rule that the CUDA path defines (the reference has no slots).
* ``oracle.model``     -- the Qwen2/Qwen3 forward of the JAX adapter
  (``src/counterfact_kv_eviction/jax_inference.py:609-637,902-1107,1156-1348,1514-1790``)
  restated in numpy with the same bfloat16 rounding points.
* ``oracle.stub_model`` -- a deterministic score source with the adapter's call
  signature, used to pin the loop logic against the reference generator.

Pinning status:
* Policies, protection wrapper and the decode/eviction loop are PINNED: the
  fixtures in ``tests/golden/`` were produced by running the reference's own,
  unmodified Python code (``tests/golden/make_golden.py``) and the CPU tests
  check this oracle against them bit for bit.
* The model forward is a restatement of JAX/XLA code that cannot run here (JAX is
  not installable in this image): its numerics are "parity unpinned" beyond the
  rounding points read from the source.  Logit/score agreement with the CUDA path
  is therefore judged with a stated bf16 tolerance.
"""
