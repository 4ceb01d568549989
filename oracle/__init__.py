"""CPU oracle for the attention hot path of zwhisper.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this package; only
`tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of
`bench.py` use it, and only as the checker or the timed CPU baseline.

Modules:
- `attention`: numpy restatement of `ops.attentionEx` (src/ops.zig:464-605 in the
  reference) in the reference's algorithm order.
- `attn_ref.c` + `cref`: the same algorithm in C with the reference's thread-pool task
  split, used as the timed CPU baseline ("port") and to cross-check the numpy restatement.
- `whisper`: synthetic audio, log-mel, ggml writer, encoder/decoder forward (the callers
  that produce real attention inputs), pinned against the reference binary's outputs.
- `qwen`: NeoX RoPE tables, transposed-key cache scatter and the GQA attention call of
  src/llm.zig:168-238.
"""
