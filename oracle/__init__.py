"""CPU oracle for the WeDLM block-parallel decode step.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (the CUDA library under
``wedlm-rs_b200/`` and its Python host mirror) imports, links or executes this
package.  Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` use it, and only as the checker or the
timed CPU reference.

The reference (arkavo-ai/WeDLM-rs) is a Rust crate whose arithmetic lives in the
unvendored ``candle`` path dependency (``Cargo.toml:10-12``, version unpinned);
neither ``cargo`` nor the candle tree is available, so the reference cannot be
built.  These modules restate, in numpy and plain C, the algorithm of the
reference files cited in each docstring.  They are pinned by:

* the reference's numpy-generated golden fixture
  (``tests/fixtures/wedlm_parity_small.json`` produced by
  ``scripts/generate_parity_fixture.py``), regenerated here by
  ``tests/golden/make_golden.py``;
* the known answers of the reference's unit tests
  (``src/decoding/sampler.rs:547-610``, ``src/decoding/reorder.rs:194-253``,
  ``src/model/rope.rs:204-246``, ``src/model/attention.rs:336-368``,
  ``src/model/mlp.rs:52-69``).

Parity for the KV-cache concat, the causal mask with a non-empty cache, entropy
values, argmax tie-breaking, the entropy-EMA cap and the streaming loop is not
covered by any reference test that runs without the real 8B checkpoint; for those
pieces the oracle follows the cited source lines and is "parity unpinned" beyond
the fixture and the unit-test known answers.
"""
