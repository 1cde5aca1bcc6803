"""Regenerate tests/golden/rust_ffi_symbols.txt: every native symbol the
reference's Rust crate declares in its `unsafe extern "C"` blocks
(src/serving/native_device.rs:1087-1207, native_mtp_device.rs:332-393,
native_qwen.rs:557-590, native_mlx.rs:574-636, native_ingestion.rs:13-14).
Those names are what a Rust build links against this library.

    QWEN_REFERENCE=<reference checkout> python tests/golden/make_ffi_list.py

The reference location comes from QWEN_REFERENCE or BASELINE.json's
"reference_path"; the committed list lets the test run without it.
"""
from __future__ import annotations

import re
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent / "rust_ffi_symbols.txt"
FILES = ["native_device.rs", "native_mtp_device.rs", "native_qwen.rs", "native_mlx.rs", "native_ingestion.rs"]


def extern_blocks(text: str):
    """Bodies of `extern "C" { ... }` blocks (brace-matched)."""
    for m in re.finditer(r'extern\s+"C"\s*\{', text):
        depth, i = 1, m.end()
        while depth and i < len(text):
            depth += {"{": 1, "}": -1}.get(text[i], 0)
            i += 1
        yield text[m.end():i - 1]


def main():
    root = O.reference_root()
    if root is None:
        raise SystemExit("reference checkout not found (set QWEN_REFERENCE)")
    names = set()
    for f in FILES:
        text = (root / "src" / "serving" / f).read_text()
        for body in extern_blocks(text):
            names.update(re.findall(r"\bfn\s+(rs_\w+)\s*\(", body))
    OUT.write_text("".join(f"{n}\n" for n in sorted(names)))
    print(f"{len(names)} symbols -> {OUT}")


if __name__ == "__main__":
    main()
