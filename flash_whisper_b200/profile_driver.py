"""Runs the hot kernels of one transcription step on representative inputs, for profiler captures.

    python -m flash_whisper_b200.profile_driver [--tokens N]

Builds a large-v3-turbo model with seeded random weights, then runs (eagerly, one launch after
another, so a profiler can select single launches by name): GPU log-mel, the 32-layer encoder
(conv GEMMs, row LayerNorm, tcgen05 GEMMs, tcgen05 attention, cross-K/V GEMM), the 4 prompt steps
and N decode steps (attention blocks, fc1, fc2, LM head). Prints the generated token ids.
"""

import argparse

import torch

from .audio import synthetic_audio
from .model import CustomModel
from .weights import TURBO, random_state_dict


@torch.inference_mode()
def main():
    parser = argparse.ArgumentParser()
    parser.add_argument('--tokens', type=int, default=4)
    args = parser.parse_args()
    model = CustomModel(state_dict=random_state_dict(0, TURBO), dims=TURBO, selftest=False, capture=False)
    model.load_audio(synthetic_audio(0, 30.0))
    model._mel()
    model._encode()
    model._prompt()
    for _ in range(args.tokens):
        model.ext.decoder_step(model.dec_desc, 1)
    torch.cuda.synchronize()
    print('tokens', model.tokens[:args.tokens + 1].tolist())


if __name__ == '__main__':
    main()
