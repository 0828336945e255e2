"""B200-native trace commitment for CommitLLM.

SHA-256 leaf hashing, Merkle trees, openings and the IO hash chain of the
reference's provider-side commit (crates/verilm-prover, crates/verilm-core
merkle.rs), run as CUDA kernels for sm_100a behind the C ABI of
``include/vcommit.h``.

* :mod:`commitllm_b200.commit` -- device runtime (contexts, KV cache views, trees)
* :mod:`commitllm_b200.verilm_rs` -- drop-in for the reference's PyO3 commit API
* :mod:`commitllm_b200.dist` -- sharding across GPUs and the root-of-roots exchange
"""
__all__ = ["commit", "verilm_rs", "dist", "build_lib"]
