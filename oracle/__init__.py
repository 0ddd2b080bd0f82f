"""CPU oracle for the PaceServe per-layer op path and KV transfer.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (``paceserve_b200``) imports
this package; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` use it, as the checker.

* ``ops_ref``     -- fp32 torch-CPU restatements of the reference formulas
                     (norms, rope + cos/sin cache, activations, the op chain).
* ``moe_ref``     -- numpy restatement of topk_softmax and moe_align_block_size.
* ``moe_align_ref.c`` -- plain-C restatement of moe_align_block_size (bit-exact
                     integer output), built to ``oracle/_build/libmoe_align_ref.so``.
* ``build_ref``   -- compiles the reference's own CUDA ops from their sources
                     into ``oracle/_ref`` (GPU oracle, run on the GPU box).
* ``kv_ref``      -- the reference's KVhelper move (per-layer gather to host,
                     index-put back), as layout oracle and timed baseline.
* ``append_ref``  -- FlashInfer's paged-KV append semantics as PaceServe calls
                     them (get_seq_lens, get_batch_indices_positions, append).
* ``compare_ref_cuda`` -- times the reference's own CUDA ops (and FlashInfer's
                     append path) beside this package's kernels on a B200.

Pinning: the moe_align restatements are pinned on CPU by the known-answer
example in the reference kernel (csrc/moe_align_block_size_kernels.cu:88-94);
every restatement is pinned against outputs of the reference's own CUDA ops
(``tests/golden/*.npz``, produced by ``tests/golden/make_golden.py`` on a B200
from ``oracle/_ref``).  ``fused_add_rms_norm``, ``gelu_and_mul``,
``gelu_tanh_and_mul`` and rope with an fp32 cache have no reference kernel:
they are pinned only by the PyTorch composition the reference performs.  The
append restatement is pinned by byte-equality with the image's FlashInfer on a
B200 (the reference pins FlashInfer 0.2.0 and does not vendor it).
"""
