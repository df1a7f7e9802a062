"""TEST INFRASTRUCTURE ONLY -- write the C shim of INTEGRATION.md (the code block
between its shim markers) to a .c file, so the oracle build can compile it
against the reference's sources and link it with the library.

  python oracle/extract_shim.py OUT.c
"""
import os
import re
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def shim_source(path=os.path.join(ROOT, "INTEGRATION.md")) -> str:
    text = open(path).read()
    m = re.search(r"<!-- shim:begin -->\s*```c\n(.*?)```\s*<!-- shim:end -->", text, flags=re.S)
    if not m:
        raise SystemExit(f"{path}: no shim block between the shim markers")
    return m.group(1)


if __name__ == "__main__":
    src = shim_source()
    out = sys.argv[1]
    os.makedirs(os.path.dirname(os.path.abspath(out)), exist_ok=True)
    with open(out, "w") as f:
        f.write(src)
