"""Write a copy of the reference's gpt2.c whose W8A8 GPU layer and token pick
run on this repository's library instead of cuBLAS (test infrastructure).

The copy replaces two line ranges of the reference file by #include lines of
this repository's own code:

  gpt2.c:1123-1331  transformer_block_gpu (with its #ifdef USE_CUDA guard)
                    -> oracle/dropin/block_w8a8.inc
  gpt2.c:2150-2245  final LayerNorm, LM head, softmax, 100 KB copy and the
                    greedy / top-k pick of the token loop
                    -> oracle/dropin/pick_w8a8.inc

Everything else (loader, buffers, KV cache, tokenizer client, token loop,
timing) is the reference's own. The line numbers belong to one version of
gpt2.c, which the SHA-256 below pins; another version is refused.

usage: python oracle/dropin_gpt2.py REF_GPT2_C OUT_C
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

SHA256 = "23dfaca1a2beaf551d7b3a9f7df55acd10465c84d6b6971596a1e23841d329b6"
HERE = Path(__file__).resolve().parent
# (first line, last line) 1-based inclusive -> replacement text
SPLICES = [
    ((1123, 1331), f'#include "{HERE / "dropin" / "block_w8a8.inc"}"\n'),
    ((2150, 2245), f'#include "{HERE / "dropin" / "pick_w8a8.inc"}"\n'),
]


def main(argv: list[str]) -> int:
    src, out = Path(argv[1]), Path(argv[2])
    data = src.read_bytes()
    if hashlib.sha256(data).hexdigest() != SHA256:
        sys.stderr.write(f"{src}: not the gpt2.c these line ranges were written for\n")
        return 1
    lines = data.decode().splitlines(keepends=True)
    for (a, b), text in sorted(SPLICES, reverse=True):
        lines[a - 1:b] = [text]
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text("".join(lines))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
