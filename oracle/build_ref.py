"""Compile the reference's host SSD server into oracle/_ref/libssd_ref.so (checker only).

The reference (monochromegane/vllm-expert-pager) keeps its C server as a string
(``_C_SOURCE`` in src/vllm_expert_pager/store.py) and compiles it at first use
with ``cc -O3 -march=native -funroll-loops -fPIC -shared -pthread``
(native.py:25).  This script reads that string from the reference's store.py,
writes it to a temporary directory outside the repository and compiles it the
same way; only the shared library lands in ``oracle/_ref/`` (git-ignored).

Usage: python oracle/build_ref.py <reference checkout or install directory>
Tests load the library, when present, to compare the reference server with
this repository's C++ server on the same request sequences.
"""

import ast
import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))


def source_of(reference: str) -> str:
    """``_C_SOURCE`` of the reference's store.py, from a checkout (``src/...``)
    or from an installed copy of the package (``pip install --target``)."""
    path = os.path.join(reference, "src", "vllm_expert_pager", "store.py")
    if not os.path.exists(path):
        path = os.path.join(reference, "vllm_expert_pager", "store.py")
    tree = ast.parse(open(path).read())
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(
            isinstance(t, ast.Name) and t.id == "_C_SOURCE" for t in node.targets
        ):
            return ast.literal_eval(node.value)
    raise SystemExit(f"no _C_SOURCE in {path}")


def build(reference: str) -> str:
    src = source_of(reference)
    out_dir = os.path.join(HERE, "_ref")
    os.makedirs(out_dir, exist_ok=True)
    out = os.path.join(out_dir, "libssd_ref.so")
    with tempfile.TemporaryDirectory() as tmp:
        c = os.path.join(tmp, "ssd.c")
        with open(c, "w") as f:
            f.write(src)
        subprocess.run([os.environ.get("CC", "cc"), "-O3", "-march=native", "-funroll-loops",
                        "-fPIC", "-shared", "-pthread", c, "-o", out, "-lm"], check=True)
    return out


if __name__ == "__main__":
    print(build(sys.argv[1]))
