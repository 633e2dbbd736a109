"""CPU oracle for the speculative draft -> verify -> accept/reject -> commit path.

TEST INFRASTRUCTURE ONLY.  This package restates, on the CPU, the algorithm of
vedantjain09/paged-speculative-engine (a pure Python / PyTorch engine) so that
the CUDA path in ``pse`` can be checked against it.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it, and only as the checker or as the timed CPU baseline.  The product
package (``pse``) never imports anything from here and has no CPU fallback.

Modules (each function cites the reference file:line it restates):

* ``model``           TinyGPT (engine/model.py) and the Llama-style model used by
                      the GQA/RoPE workload (no reference counterpart; restated
                      in TinyGPT's style with the same forward contract).
* ``paged_cache``     BlockAllocator / PagedKVCache (engine/paged_cache.py).
* ``batched_forward`` batched_forward_append (engine/batched_forward.py).
* ``sampling``        softmax / multinomial / argmax helpers (engine/sampling.py)
                      plus inverse-CDF sampling from an explicit uniform.
* ``speculative``     prefill_request / batched_speculative_step
                      (engine/speculative.py), with an explicit-uniform mode.
* ``scheduler``       run_continuous_speculative_batches (engine/scheduler.py).
* ``generate``        generate_naive / generate_cached / speculative_generate_batched
                      (engine/generate.py).
* ``accept``          vectorised numpy statement of the accept/resample rule with
                      explicit uniforms, in the arithmetic the CUDA kernel uses.
* ``alloc``           batched (prefix-scan) restatement of the LIFO free list.
* ``attention``       paged attention over a block pool (engine/model.py:99-116
                      applied to engine/paged_cache.py's layout).
* ``philox``          Philox4x32-10 counter-based generator (Salmon et al. 2011).
* ``tree``            tree speculation (b candidate branches per step; the
                      reference's README future work), b = 1 being the linear step.

Parity pin: ``tests/golden/`` holds vectors produced by running the reference
itself (script ``tests/golden/make_golden.py``); ``tests/test_oracle_golden.py``
checks this oracle against them.
"""
