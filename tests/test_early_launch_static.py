"""A kernel launched early (launch_pdl: programmatic stream serialisation) may
start while the previous kernel on the stream is still running, so it must
execute pdl_wait() before it touches global memory, or it could read that
kernel's outputs before they are written.  This reads the CUDA sources and
checks that every kernel passed to launch_pdl calls pdl_wait() in its body
(where in the body is checked by tests/test_gpu_dependent_chain.py, which runs
chains of dependent ops back to back against the same chains synchronised
after every op)."""
import re
from pathlib import Path

CSRC = Path(__file__).resolve().parents[1] / "bee_b200" / "csrc"


def _launched_early():
    names = set()
    for f in CSRC.glob("*.cu"):
        for m in re.finditer(r"launch_pdl\(\s*([A-Za-z_]\w*)", f.read_text()):
            names.add((f.name, m.group(1)))
    return names


def _resolve(text, name):
    """`auto k = kernel<...>; launch_pdl(k, ...)` names the kernel through a local."""
    m = re.search(r"auto\s+" + re.escape(name) + r"\s*=\s*([A-Za-z_]\w*)\s*<", text)
    return m.group(1) if m else name


def _kernel_body(text, name):
    m = re.search(r"__global__[^;{]*?\b" + re.escape(name) + r"\s*\(", text)
    if not m:
        return None
    i = text.index("{", m.end())
    depth = 0
    for j in range(i, len(text)):
        depth += {"{": 1, "}": -1}.get(text[j], 0)
        if depth == 0:
            return text[i:j + 1]
    raise AssertionError(f"unbalanced braces in {name}")


def _bodies():
    for fname, name in sorted(_launched_early()):
        text = (CSRC / fname).read_text()
        kernel = _resolve(text, name)
        body = _kernel_body(text, kernel)
        if body is None:  # defined in a header
            for h in sorted(CSRC.glob("*.cuh")):
                body = _kernel_body(h.read_text(), kernel)
                if body is not None:
                    break
        assert body is not None, f"{fname}: kernel {kernel} not found"
        yield fname, kernel, body


def test_every_early_launched_kernel_waits():
    found = list(_bodies())
    assert len(found) >= 15, [k for _, k, _ in found]
    missing = [f"{f}: {k}" for f, k, b in found if "pdl_wait()" not in b]
    assert not missing, "launched early without pdl_wait(): " + ", ".join(missing)

