"""CPU oracle for the activation-sparse GPT-NeoX MLP — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference's algorithm for the hot path
(thiagocmattar/sparsity-spillover):

* gates        src/sparsity_research/sites.py:86-107 (one-sided / symmetric
               thresholds), sites.py:218-226 (ReLU via build_gate), and the
               corner-tile gate runs/063-2026-10-07-pythia14m-tile-specialized-kernel/tile_gate.py:20-33;
* the MLP      transformers GPTNeoXMLP.forward with ``act`` replaced by a gate
               (src/sparsity_research/pythia.py:76-77);
* tile bits    the OR-reduction of the gate's element mask over 16x64 tiles and
               the issued/bypassed MMA accounting of
               runs/042-2026-09-20-pythia70m-sparse-scale/tile_oracle.py:4-20;
* the head     runs/068-2026-10-08-pythia14m-aligned-vocabulary-tiles/inference/head.cu:9-16
               (fp32 corner certificates) and head.py:31-37 (weight packing).

It is pinned against golden vectors produced by the reference's own modules
(tests/golden/make_golden.py).  Only ``tests/``, ``__graft_entry__.smoke`` and the
CPU-baseline leg of ``bench.py`` may import it, and only as the checker or the
timed reference arm — never as part of the product's compute path.
"""
