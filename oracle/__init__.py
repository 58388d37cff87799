"""CPU oracle for the B200 encoder engine — TEST INFRASTRUCTURE ONLY.

A numpy restatement of sam3.cpp's hot-path graph builders (PABannier/sam3.cpp),
used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the
checker. Nothing in the product (sam3.cpp_b200/) imports it.

Pinning: the block formats (quant.py) are pinned bit-exactly to gguf-py 0.19.0
(an independent implementation of ggml's quantisers); the ViT + SimpleFPN
forward (vit.py) and memory attention (mem_attn.py) are pinned to outputs of
the reference's own PyTorch dump code (tests/dump_vit_reference.py,
tests/dump_phase7_reference.py) run on seeded synthetic checkpoints, stored as
fixtures in tests/golden/. The ggml CPU kernels themselves are not available
here (the ggml submodule is not vendored), so parity to ggml's exact rounding
is unpinned; the Hiera forward (hiera.py) is pinned only through its shared
components (window partition, RoPE tables, PE, LayerNorm, attention).
"""
