"""CPU oracle for the Fracture elementwise + TurboQuant hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product path (the ``fracture_b200``
package and its CUDA library) imports, links or calls anything in this
directory. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` use it, and only as the checker or as the timed CPU
reference, never as the thing being measured or shipped.

Contents
--------
``ops``        numpy restatement of the reference's elementwise kernels
               (embedding, add, rmsnorm, rope, silu_mul) and of the RoPE
               frequency precompute, plus the llama3 frequency rule.
``turboquant`` restatement of ``crates/fracture-core/src/turboquant.rs``
               (Lloyd-Max solver, Haar rotation generator, config helpers) and
               of the compress / decompress arithmetic, plus the paged
               quantized KV cache write of
               ``crates/fracture-engine/src/quantized_paged_kv_cache.rs``.
``refio``      reader/writer for the reference's tensor ``.bin`` format.
``cpu_chain``  the reference's PyTorch-CPU numerical path for the per-layer op
               chain, used as the timed CPU baseline.
``tq_oracle.c`` C version of the exact TurboQuant compress arithmetic
               (sequential non-fused float32 sums), built by ``oracle/Makefile``
               into ``oracle/_build/libtq_oracle.so``.

Parity pins (what the oracle itself is checked against) are listed in
``tests/test_oracle_golden.py`` and ``tests/test_oracle_turboquant.py``.
"""
