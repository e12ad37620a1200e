"""flash_whisper_b200: batch-1 Whisper-large-v3-turbo hot path for NVIDIA B200 (sm_100a).

Hand-written CUDA kernels behind a C ABI (include/flash_whisper.h, libflashwhisper.so), with a thin
PyTorch host layer that keeps the call surface of the reference's custom/ext.py and custom/model.py:
`flash_whisper_b200.ext.load_ext()` and `flash_whisper_b200.model.CustomModel`.
"""

__version__ = '0.1.0'
