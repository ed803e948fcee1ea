"""Build step for the reference-kernel checker (test infrastructure only).

Cuts the CUDA C source of the reference's persistent subtree kernels -- the
raw string constant ``GPU_PERSISTENT_SUBTREE_KERNEL_SRC`` of
shear-core/src/algorithm/pipnn/compute_backend.rs (lines 4840-17381 at the
surveyed revision) -- out of the reference checkout and writes it, unchanged,
to ``oracle/_ref/ref_persistent_subtree.cu``.  The reference compiles the same
text at run time with NVRTC (compute_backend.rs:22303-22404); here nvcc
compiles it for sm_100a beside ``ref_harness.cu``.

The extracted text is never committed (``oracle/_ref/`` is git-ignored); only
the built shared libraries travel to the GPU box.  Usage:

    python extract_ref_kernels.py <reference root> <output .cu>
"""
from __future__ import annotations

import hashlib
import os
import sys

SOURCE = os.path.join("shear-core", "src", "algorithm", "pipnn", "compute_backend.rs")
OPEN = 'pub(super) const GPU_PERSISTENT_SUBTREE_KERNEL_SRC: &str = r#"'
CLOSE = '"#;'


def extract(reference_root: str) -> str:
    path = os.path.join(reference_root, SOURCE)
    with open(path, "r", encoding="utf-8") as f:
        text = f.read()
    start = text.find(OPEN)
    if start < 0:
        raise SystemExit(f"kernel string constant not found in {path}")
    start += len(OPEN)
    end = text.find("\n" + CLOSE, start)
    if end < 0:
        raise SystemExit(f"end of the kernel string constant not found in {path}")
    # A Rust raw string (r#"..."#) carries its text verbatim: no escapes to undo.
    return text[start:end + 1]


def main(argv) -> int:
    if len(argv) != 3:
        print(__doc__)
        return 2
    body = extract(argv[1])
    os.makedirs(os.path.dirname(os.path.abspath(argv[2])), exist_ok=True)
    tmp = argv[2] + ".tmp"
    with open(tmp, "w", encoding="utf-8") as f:
        f.write(body)
    os.replace(tmp, argv[2])
    digest = hashlib.sha256(body.encode("utf-8")).hexdigest()
    print(f"extracted {body.count(chr(10))} lines, sha256 {digest[:16]}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
