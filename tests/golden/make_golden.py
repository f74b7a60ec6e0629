"""Writes the golden vectors the parity tests pin against, from the reference repository's own test data.

Run once in a checkout that has the reference next to it:
    python tests/golden/make_golden.py /path/to/reference

Inputs (read as text, nothing is executed):
  tests/fixtures/llama-cpp-reference.txt  llama.cpp (llama-cpp-python 0.3.36, CPU) outputs for the tiny models of
                                          tests/TinyModels.cs StandardSpecs(): the argmax at each of the 12 probe
                                          positions and the logits at the last position (4 decimals).
Output:
  tests/golden/llamacpp_reference.json    {"models": {key: {"argmax": [...], "last": [...]}}, "probe_tokens": [...]}

The reference's tolerance for these (tests/Tests.cs:250-278): max|d|/std <= 0.02 for f32/f16 and 0.2 for quantized
weights, with the top token agreeing at >= T-1 of the 12 positions.
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PROBE_TOKENS = [1, 10, 50, 100, 200, 257, 290, 5, 7, 99, 33, 72]   # tests/TinyModels.cs:187


def main(ref_root):
    path = os.path.join(ref_root, "tests", "fixtures", "llama-cpp-reference.txt")
    models, cur = {}, None
    with open(path, encoding="utf-8") as f:
        for line in f:
            line = line.rstrip("\n")
            if line.startswith("model "):
                cur = line.split(" ", 1)[1].strip()
                models[cur] = {}
            elif line.startswith("argmax ") and cur:
                models[cur]["argmax"] = [int(v) for v in line.split()[1:]]
            elif line.startswith("last ") and cur:
                models[cur]["last"] = [float(v) for v in line.split()[1:]]
    out = {"source": "tests/fixtures/llama-cpp-reference.txt (llama-cpp-python 0.3.36, CPU)",
           "probe_tokens": PROBE_TOKENS, "models": models}
    with open(os.path.join(HERE, "llamacpp_reference.json"), "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print(f"wrote {len(models)} models")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference")
    main(sys.argv[1])
