"""Generate the golden fixtures in this folder from the reference's own shipped binary.

Run in the build container, where the read-only reference tree (with its prebuilt
`zig-out-safe/bin/zwhisper`) is available:

    python tests/golden/make_golden.py /path/to/reference

It writes a synthetic tiny.en-shaped ggml model (seeded, N(0, 0.02^2) f16 weights) and
30 s of the seeded synthetic audio to a temporary folder, runs the binary's `mel` and
`logits` commands (src/main.zig:173-191: the whole encoder, then one decoder step on
[sot]), and stores small samples of both outputs in whisper_tiny_synth.npz. The tests
rebuild the same model and audio from the seeds and compare the oracle (and the GPU path)
against these numbers; they never run the binary.
"""
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import whisper as W  # noqa: E402

MODEL_SEED = 0
AUDIO_SEED = 0
MEL_FRAME_STEP = 29
LOGIT_STEP = 16


def main(ref_root: str) -> None:
    binary = os.path.join(ref_root, "zig-out-safe", "bin", "zwhisper")
    hp = W.TINY_EN
    with tempfile.TemporaryDirectory() as tmp:
        model = os.path.join(tmp, "tiny_synth.bin")
        wav = os.path.join(tmp, "synth30.wav")
        W.write_ggml(model, hp, W.synth_model(hp, seed=MODEL_SEED), W.mel_filters(80))
        W.write_wav(wav, W.synth_audio(30.0, seed=AUDIO_SEED))
        mel_out = os.path.join(tmp, "mel.f32")
        logits_out = os.path.join(tmp, "logits.f32")
        r1 = subprocess.run([binary, "mel", model, wav, mel_out], capture_output=True, text=True, check=True)
        r2 = subprocess.run([binary, "logits", model, wav, logits_out], capture_output=True, text=True, check=True)
        mel = np.fromfile(mel_out, np.float32).reshape(80, -1)
        logits = np.fromfile(logits_out, np.float32)
    top = np.argsort(-logits)[:64]
    np.savez_compressed(
        os.path.join(HERE, "whisper_tiny_synth.npz"),
        mel_frames=np.arange(0, mel.shape[1], MEL_FRAME_STEP),
        mel_sample=mel[:, ::MEL_FRAME_STEP],
        mel_shape=np.array(mel.shape),
        logits_idx=np.arange(0, logits.size, LOGIT_STEP),
        logits_sample=logits[::LOGIT_STEP],
        logits_top_idx=top,
        logits_top=logits[top],
        logits_sum=np.float64(logits.astype(np.float64).sum()),
        logits_sumsq=np.float64((logits.astype(np.float64) ** 2).sum()),
        argmax=np.int64(logits.argmax()),
        n_vocab=np.int64(logits.size),
        seeds=np.array([MODEL_SEED, AUDIO_SEED]),
        binary_mel_line=np.array(r1.stdout.strip()),
        binary_logits_line=np.array(r2.stdout.strip()),
    )
    print(r1.stdout.strip())
    print(r2.stdout.strip())


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference")
    main(sys.argv[1])
