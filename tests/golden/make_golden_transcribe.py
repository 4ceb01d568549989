"""Generate tests/golden/whisper_tiny_transcribe.json from the reference's shipped binary.

Run in the build container, where the read-only reference tree (with its prebuilt
`zig-out-safe/bin/zwhisper`) is available:

    python tests/golden/make_golden_transcribe.py /path/to/reference

It writes the seeded synthetic tiny.en model (the one make_golden.py uses) and seeded
synthetic audio to a temporary folder, runs the binary's `transcribe ... --json
--no-voices` (src/main.zig:193-229: greedy long-form decoding with whisper.cpp's timestamp
rules, src/transcribe.zig:248-580) and stores every segment it prints (start, end,
token ids, text) for two cases: 30 s without the previous-window prompt, and 95 s (four
windows) with it. The tests rebuild the model and audio from the seeds and never run the
binary.
"""
import json
import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import whisper as W  # noqa: E402

MODEL_SEED = 0
AUDIO_SEED = 0
CASES = [
    {"name": "30s_no_context", "seconds": 30.0, "context": False},
    {"name": "95s_context", "seconds": 95.0, "context": True},
]


def main(ref_root: str) -> None:
    binary = os.path.join(ref_root, "zig-out-safe", "bin", "zwhisper")
    hp = W.TINY_EN
    out = {"model_seed": MODEL_SEED, "audio_seed": AUDIO_SEED, "model": "synthetic tiny.en (oracle.whisper.synth_model)",
           "cases": []}
    with tempfile.TemporaryDirectory() as tmp:
        model = os.path.join(tmp, "tiny_synth.bin")
        W.write_ggml(model, hp, W.synth_model(hp, seed=MODEL_SEED), W.mel_filters(80))
        for case in CASES:
            wav = os.path.join(tmp, f"{case['name']}.wav")
            W.write_wav(wav, W.synth_audio(case["seconds"], seed=AUDIO_SEED))
            args = [binary, "transcribe", model, wav, "--json", "--no-voices", "-t", "8"]
            if not case["context"]:
                args.append("--no-context")
            r = subprocess.run(args, capture_output=True, text=True, check=True)
            segs = [json.loads(line) for line in r.stdout.splitlines() if line.startswith("{")]
            out["cases"].append({**case, "binary_summary": r.stderr.strip().splitlines()[-1],
                                 "segments": [{"t0": s["t0"], "t1": s["t1"], "tokens": s["tokens"], "text": s["text"]}
                                              for s in segs]})
            print(case["name"], len(segs), "segments")
    with open(os.path.join(HERE, "whisper_tiny_transcribe.json"), "w") as f:
        json.dump(out, f, separators=(",", ":"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden_transcribe.py /path/to/reference")
    main(sys.argv[1])
