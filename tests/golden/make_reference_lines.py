"""Writes tests/golden/reference_lines.json: the line count of every reference source
file that this repository cites (file:line), and the line on which each exported
function / constant / interface of those files starts.

Run it where the reference project is checked out (it only reads text files):

    python tests/golden/make_reference_lines.py /path/to/reference

tests/test_citations.py checks every citation in the repository against this
fixture, so the check runs without the reference present.
"""
import json
import os
import re
import sys

FILES = ["src/core/engine.ts", "src/core/gpu.ts", "src/core/gguf.ts", "src/core/pager.ts", "src/core/quant.ts",
         "src/core/shaders.ts", "src/core/qwen-shaders.ts", "src/core/context.ts", "src/core/source.ts",
         "src/core/bpe.ts", "src/core/gpt2-tokenizer.ts", "src/core/tokenizer.ts", "src/core/qwen-tokenizer.ts",
         "src/sdk.ts", "src/worker.ts", "src/verify.ts", "src/verify-context.ts", "src/verify-qwen.ts",
         "scripts/verify-dense.mjs", "tests/quant.test.ts", "tests/context.test.ts", "tests/model-config.test.ts",
         "tests/pager.test.ts", "tests/gguf.test.ts", "tests/source.test.ts", "tests/tokenizer.test.ts",
         "tests/gpt2-tokenizer.test.ts", "tests/qwen-tokenizer.test.ts"]
SYMBOL = re.compile(r"^export\s+(?:async\s+)?(?:function\*?|const|class|interface|type)\s+([A-Za-z0-9_]+)")


def main(root: str) -> None:
    out = {}
    for rel in FILES:
        path = os.path.join(root, rel)
        if not os.path.exists(path):
            continue
        lines = open(path, encoding="utf-8", errors="replace").read().split("\n")
        if lines and lines[-1] == "":
            lines.pop()
        symbols = {}
        for i, line in enumerate(lines, 1):
            m = SYMBOL.match(line)
            if m:
                symbols[m.group(1)] = i
        out[rel] = {"lines": len(lines), "symbols": symbols}
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_lines.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print(f"wrote {dst}: {len(out)} files")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
