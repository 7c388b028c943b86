"""Build step for the reference checker (TEST INFRASTRUCTURE ONLY).

Copies, verbatim and unmodified, plain-C++ helpers of the reference out of
files that as a whole need the vpipe SDK or Metal (so cannot be compiled
here) into oracle/_ref/ (git-ignored, never committed), where
oracle/ref_harness.cc compiles them beside shim types:

  dit   src/ltx25-dit.cc: bf16_to_f32_, f32_to_bf16_, gemv_host_,
        lora_gemv_host_, silu_, timestep_sinusoid_ -- the host adaLN chain's
        arithmetic (src/ltx25-dit.cc:30-135)
  lora  tests/ltx25-lora-apply-test.cc: struct HostPair and fold (W += B A,
        lines 330-366), the reference's CPU fold of an adapter;
        src/ltx25-lora.cc: bf16_to_f32_, f32_to_bf16_ (the rounding its
        scaled_ uses to fold the adapter factor into A, lines 27-47)

usage: python3 extract_ref_helpers.py <reference tree> <out dir>
"""
import os
import re
import sys

JOBS = {
    "ref_dit.inc": ("src/ltx25-dit.cc",
                    ["bf16_to_f32_", "f32_to_bf16_", "gemv_host_", "lora_gemv_host_",
                     "silu_", "timestep_sinusoid_"]),
    "ref_lora_test.inc": ("tests/ltx25-lora-apply-test.cc", ["struct HostPair", "fold"]),
    "ref_lora_bits.inc": ("src/ltx25-lora.cc", ["bf16_to_f32_", "f32_to_bf16_"]),
}


def block_end(src: str, brace: int) -> int:
    depth = 0
    for i in range(brace, len(src)):
        if src[i] == "{":
            depth += 1
        elif src[i] == "}":
            depth -= 1
            if depth == 0:
                return i
    raise SystemExit("extract_ref_helpers: unbalanced braces")


def extract(src: str, name: str, path: str) -> str:
    if name.startswith("struct "):
        m = re.search(r"^" + re.escape(name) + r"\s*\{", src, re.M)
        if m is None:
            raise SystemExit(f"extract_ref_helpers: '{name}' not found in {path}")
        end = block_end(src, m.end() - 1)
        semi = src.index(";", end)
        return src[m.start():semi + 1]
    # return type on its own line, then `name(args...)` at column 0
    m = re.search(r"^([A-Za-z_:<>0-9 ]+)\n" + re.escape(name) + r"\(", src, re.M)
    if m is None:
        raise SystemExit(f"extract_ref_helpers: '{name}' not found in {path}")
    return src[m.start():block_end(src, src.index("{", m.end())) + 1]


def main() -> None:
    ref, out_dir = sys.argv[1], sys.argv[2]
    os.makedirs(out_dir, exist_ok=True)
    for out, (rel, names) in JOBS.items():
        path = os.path.join(ref, rel)
        with open(path, "r", encoding="utf-8") as f:
            src = f.read()
        parts = [f"// extracted from {rel} by oracle/extract_ref_helpers.py\n"]
        for name in names:
            parts.append(extract(src, name, rel) + "\n\n")
        with open(os.path.join(out_dir, out), "w", encoding="utf-8") as f:
            f.write("".join(parts))


if __name__ == "__main__":
    main()
