"""CPU oracle for the indexed sparse gated-FFN hot path -- TEST INFRASTRUCTURE ONLY.

A restatement of the reference algorithm (robjlyons/qwen-contextual-compression)
used as the checker: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` may import it.  The product package never does;
it has no CPU fallback.

* ``oracle.ffn``    -- dynamic sparse FFN (runtime/ffn.py:20-43), scatter
                      reconstruct and importance scores (oracle/sparse_ffn.py,
                      oracle/importance.py), the packed record layout, an fp64
                      numpy formulation for tolerance headroom.
* ``oracle.select`` -- top-K with the fixed tie rule, block top-K, unions.
* ``oracle.lru``    -- the LRU neuron-cache accounting of runtime/temporal.py:55-75.

Pinned by the golden vectors in ``tests/golden`` (made by running the
reference itself, ``tests/golden/make_golden.py``).
"""
