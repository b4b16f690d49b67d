"""CPU oracle for the BFP SmolLM2-135M decode path -- TEST INFRASTRUCTURE ONLY.

This package is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product (``bfp200``) never imports,
links or executes anything in here; it fails loudly when its CUDA library is
missing instead of falling back to this code.

Contents
--------
bfp_oracle  numpy restatement of the reference's bit-exact BFP simulator
            (rtl/vc707/host/gen_smollm_blockfp_full.py), function by function.
synth       seeded synthetic SmolLM2-135M model whose float weights are fixed
            points of BFP decode(quantize(.)), so the packed image and the
            simulator see identical values.

Pinning: the restatement is checked against fixtures produced by running the
reference's own functions (tests/golden/make_golden.py, run in a container
that has the reference checked out) -- see tests/test_oracle.py.
"""
