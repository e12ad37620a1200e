"""Times the reference's CUDA backend (re-hosted by oracle/ref_pipeline.py: its kernels compiled from
source, HF fp16 encoder with SDPA, cuBLAS projections, CUDA graphs) and this package on the same GPU,
same seeded weights and audio, 224 forced tokens. Not collected by pytest (test infrastructure run by
hand on a GPU box):

    python tests/time_reference_backend.py

Prints E2E (host timer around transcribe, median of 5), encoder and decode stage times and the
decode step time per token (8-step CUDA graph replays, CUDA events), and whether the token ids match.
"""

import statistics
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from flash_whisper_b200.audio import synthetic_audio  # noqa: E402
from flash_whisper_b200.model import CustomModel  # noqa: E402
from flash_whisper_b200.weights import TURBO, random_state_dict  # noqa: E402
from oracle.ref_pipeline import RefCudaBackend  # noqa: E402

N_TOKENS = 224


def per_token_us(replay, steps, iters=20):
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        replay()
    torch.cuda.synchronize()
    a.record()
    for _ in range(iters):
        replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / (iters * steps)


@torch.inference_mode()
def main():
    sd = random_state_dict(0, TURBO)
    audio = synthetic_audio(0, 30.0)
    ref = RefCudaBackend(sd, TURBO)
    for _ in range(2):
        ref.transcribe(audio, N_TOKENS)
    runs = [ref.transcribe(audio, N_TOKENS) for _ in range(5)]
    ref_tokens = runs[0][0]
    med = lambda k: statistics.median(r[1][k] for r in runs) * 1e3  # noqa: E731
    print('reference CUDA backend: e2e %.2f ms, mel %.3f ms, encoder %.3f ms, decode %.2f ms, %.1f us/token' % (
        med('e2e_s'), med('mel_s'), med('encoder_s'), med('decode_s'), per_token_us(ref.graph_chunk.replay, 8)))
    del ref
    torch.cuda.empty_cache()
    model = CustomModel(state_dict=sd, dims=TURBO, selftest=False)
    for _ in range(2):
        model.transcribe(audio, max_new_tokens=N_TOKENS, stop_at_eos=False)
    outs = [model.transcribe(audio, max_new_tokens=N_TOKENS, stop_at_eos=False) for _ in range(5)]
    print('flash_whisper_b200:     e2e %.2f ms, %.1f us/token' % (
        statistics.median(o['e2e_s'] for o in outs) * 1e3, per_token_us(model.run_chunk, model.chunk)))
    print('token ids identical:', outs[0]['token_ids'] == ref_tokens[:N_TOKENS])


if __name__ == '__main__':
    main()
