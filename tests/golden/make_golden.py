#!/usr/bin/env python3
"""Regenerate the golden fixtures in this directory from the reference's own
fixture generators (eating-and-drinking/slate `tools/*.py`).

Those scripts write hard-coded `/tmp/slate_*` paths.  This driver runs each of
them unmodified with `builtins.open` redirected so that every `/tmp/<name>`
they write lands here as `<name>` instead; nothing is written outside this
directory.  The reference tree is only needed when regenerating (it is absent
on GPU hosts; the committed fixtures are what the tests read).

Fixtures produced (reference script -> files):
  tools/make_q4k_test.py           -> slate_q4k_test.bin   (1 Q4_K block, originals, recon)
  tools/make_q4k_gguf.py           -> slate_q4k.gguf, slate_q4k_expected.f32 (16x256 Q4_K)
  tools/make_rope_ref.py           -> slate_rope_ref.bin
  tools/make_tiny_llama_gguf.py    -> slate_tiny_llama.gguf (f32 MHA, D=32)
  tools/make_llama_ref.py          -> slate_llama_ref.bin (numpy logits for the above)
  tools/make_tiny_llama_gqa_gguf.py-> slate_tiny_llama_gqa.gguf, slate_tiny_llama_gqa_ref.bin
  tools/make_tiny_llama_q4k_gguf.py-> slate_tiny_llama_q4k.gguf, slate_tiny_llama_q4k_ref.bin

Usage: python tests/golden/make_golden.py [REFERENCE_ROOT]
"""
import builtins
import hashlib
import os
import runpy
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SCRIPTS = [
    "make_q4k_test.py",
    "make_q4k_gguf.py",
    "make_rope_ref.py",
    "make_tiny_llama_gguf.py",
    "make_llama_ref.py",
    "make_tiny_llama_gqa_gguf.py",
    "make_tiny_llama_q4k_gguf.py",
]


def main() -> None:
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get(
        "SLATE_REFERENCE_ROOT", "")
    if not ref_root or not os.path.isdir(os.path.join(ref_root, "tools")):
        sys.exit("usage: make_golden.py REFERENCE_ROOT (the slate source tree)")
    real_open = builtins.open

    def redirect(path, *a, **kw):
        if isinstance(path, str) and path.startswith("/tmp/"):
            path = os.path.join(HERE, os.path.basename(path))
        return real_open(path, *a, **kw)

    builtins.open = redirect
    saved_argv = sys.argv
    try:
        for name in SCRIPTS:
            sys.argv = [name]          # scripts default their output path to /tmp
            runpy.run_path(os.path.join(ref_root, "tools", name), run_name="__main__")
    finally:
        builtins.open = real_open
        sys.argv = saved_argv
    with real_open(os.path.join(HERE, "SHA256SUMS"), "w") as f:
        for fn in sorted(os.listdir(HERE)):
            if fn.endswith((".bin", ".gguf", ".f32")):
                h = hashlib.sha256(real_open(os.path.join(HERE, fn), "rb").read()).hexdigest()
                f.write(f"{h}  {fn}\n")


if __name__ == "__main__":
    main()
