"""Generate tests/golden/blackwell_binding.json: every downcall descriptor the
reference's FFM class declares for libaljabr_blackwell.so.

Source: backend/blackwell/aljabr-kernel-blackwell/src/main/java/tech/kayys/
aljabr/blackwell/binding/BlackwellBinding.java, method bindAll() (:456-583).
Each `bind(FN_X, FunctionDescriptor.of(RET, ARGS...))` or
`FunctionDescriptor.ofVoid(ARGS...)` becomes one entry

    symbol -> {"ret": "JAVA_INT" | "JAVA_LONG" | "ADDRESS" | "void",
               "args": ["ADDRESS", "JAVA_INT", ...], "line": <bind line>}

with FN_X resolved through the class's `FN_X = "aljabr_blackwell_..."`
constants.  The JSON is committed, so the ABI test needs no reference tree;
rerun this script (with the reference mounted) to refresh it:

    python tests/golden/make_binding.py /path/to/reference
"""
from __future__ import annotations

import json
import os
import re
import sys

REL = ("backend/blackwell/aljabr-kernel-blackwell/src/main/java/tech/kayys/aljabr/blackwell/binding/"
       "BlackwellBinding.java")


def parse(text: str) -> dict:
    names = dict(re.findall(r'static final String (FN_\w+)\s*=\s*"(aljabr_blackwell_\w+)"', text))
    start = text.index("private void bindAll()")
    body = text[start:]
    out = {}
    for m in re.finditer(r"bind\((FN_\w+),\s*FunctionDescriptor\.(of|ofVoid)\((.*?)\)\);", body, flags=re.S):
        fn, kind, args = m.group(1), m.group(2), m.group(3)
        layouts = re.findall(r"ValueLayout\.(\w+)", args)
        if kind == "of":
            ret, params = layouts[0], layouts[1:]
        else:
            ret, params = "void", layouts
        line = text[:start + m.start()].count("\n") + 1
        out[names[fn]] = {"ret": ret, "args": params, "line": line}
    return out


def main(ref_root: str) -> None:
    with open(os.path.join(ref_root, REL)) as f:
        table = parse(f.read())
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "blackwell_binding.json")
    with open(dst, "w") as f:
        json.dump({"source": REL + " bindAll()", "descriptors": table}, f, indent=1, sort_keys=True)
        f.write("\n")
    print(f"{len(table)} descriptors -> {dst}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_binding.py <reference project root>")
    main(sys.argv[1])
