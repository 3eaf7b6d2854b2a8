"""CPU oracle for the vllm_apple paged-attention hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
legs of ``bench.py`` may use it, and only as the checker or as the timed
reference CPU implementation.

Contents
--------
``paged_attention``  numpy restatement of every function on the path
                     (KV-cache scatter, decode attention, token-parallel
                     prefill attention, RMSNorm, Neox/GPT-J RoPE, SiLU-mul),
                     each citing the reference file:line it follows.
``mps_port``         torch-CPU restatement of the reference's pure-PyTorch
                     attention backend (``MPSAttentionImpl``), the reference's
                     own CPU code path, used as the timed CPU baseline.
``kv_scatter.c``     plain-C restatement of the reference's native KV writer,
                     built by ``oracle/Makefile`` into ``oracle/_build``.
``Makefile``         also compiles the reference's own ``kv_write.c`` (when the
                     reference tree is present) into ``oracle/_ref``.

Parity pinning: the numpy restatement is checked against golden vectors in
``tests/golden/`` that were produced by running the reference's own PyTorch
path and its own numpy RoPE-table code (``tests/golden/make_golden.py``), and
against the reference's compiled ``kv_write.c``.
"""
