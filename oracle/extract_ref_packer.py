"""Build step for the reference checker (TEST INFRASTRUCTURE ONLY).

The reference's only w8g64 packer is the `quantize()` helper inside
tests/ltx25-qlinear-test.cc (lines 94-141), next to `to_bf16`/`from_bf16`
(lines 66-81).  That file as a whole needs the vpipe SDK and Metal, so it
cannot be compiled here; the three functions themselves are plain C++.
This script copies those three function bodies, verbatim and unmodified,
from the reference tree into oracle/_ref/ref_packer.inc (git-ignored, never
committed), where oracle/ref_harness.cc compiles them.  The output is the
reference's own code, used only to pin oracle/ltx_oracle.c.

usage: python3 extract_ref_packer.py <ltx25-qlinear-test.cc> <out.inc>
"""
import re
import sys

WANT = ("to_bf16", "from_bf16", "quantize")


def extract(src: str, name: str) -> str:
    # The reference writes the return type on its own line, then
    # `name(args...)` at column 0, then the brace-delimited body.
    m = re.search(r"^([A-Za-z_:<>0-9 ]+)\n" + re.escape(name) + r"\(", src, re.M)
    if m is None:
        raise SystemExit(f"extract_ref_packer: '{name}' not found")
    start = m.start()
    brace = src.index("{", m.end())
    depth = 0
    for i in range(brace, len(src)):
        if src[i] == "{":
            depth += 1
        elif src[i] == "}":
            depth -= 1
            if depth == 0:
                return src[start:i + 1]
    raise SystemExit(f"extract_ref_packer: unbalanced braces in '{name}'")


def main() -> None:
    src_path, out_path = sys.argv[1], sys.argv[2]
    with open(src_path, "r", encoding="utf-8") as f:
        src = f.read()
    parts = [f"// extracted from {src_path} by oracle/extract_ref_packer.py\n"]
    for name in WANT:
        parts.append(extract(src, name) + "\n\n")
    with open(out_path, "w", encoding="utf-8") as f:
        f.write("".join(parts))


if __name__ == "__main__":
    main()
