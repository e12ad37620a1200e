"""Parity oracle for flash_whisper_b200 — TEST INFRASTRUCTURE, NOT PART OF THE PRODUCT.

A CPU restatement (numpy / float64 where it matters) of the reference's batch-1 Whisper path:
custom/kernels/whisper_kernels.cu (the four decode kernels), custom/model.py (_log_mel, _step,
_encode, transcribe) and custom/pytorch_model.py (the greedy loop), plus the transformers code the
reference calls (feature_extraction_whisper.py, modeling_whisper.py). Each function cites the
reference file:line it follows.

Pinning: kernels.py / model_np.py are checked in tests/ against golden vectors that
tests/golden/make_golden.py produced by running the reference's own Python (custom/model.py's
_log_mel, custom/selftest.py's _attention_ref) and transformers' WhisperFeatureExtractor /
WhisperForConditionalGeneration in the build container. build_ref.py compiles the reference's own
CUDA kernels from their source into oracle/_ref/ so GPU tests can compare against them.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / `--impl reference` legs may
import this package. The product (flash_whisper_b200/) never does.
"""
