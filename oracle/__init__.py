"""CPU oracle of the PP-OCRv6 hot path -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg,
and only as the checker or the timed CPU baseline; the product path
(ppocr-rs_b200/) never imports it.

Parity status: model-level parity is UNPINNED against execution of the
reference.  The reference is Rust (no Rust toolchain in this image) and its
GPU path is wgpu/Vulkan (no graphics stack), so neither of its backends can
run here.  The restatement is pinned by the reference's own known-answer
tests (erf values, rank-one factorisation, intraclass fusion, upsample order,
linear+softmax, ConvT layout, pooling, preprocessing, CTC decoding), which
tests/test_oracle.py re-expresses, and frozen by the golden fixtures under
tests/golden/ that tests/test_golden.py re-derives.
"""
