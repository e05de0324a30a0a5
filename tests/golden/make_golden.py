"""Writes the golden fixtures of this directory from the CPU oracle.

    python tests/golden/make_golden.py            # all cases
    python tests/golden/make_golden.py attention  # one case

For every case of tests/golden_cases.py: <case>.npz holds its small output
arrays, and digests.json holds the SHA-256 digests of its seeded inputs
("<case>/input/<name>") and of its large outputs ("<case>/<name>").
Regenerate only after a deliberate change to the oracle's arithmetic, and
say why in the commit."""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
TESTS = os.path.dirname(HERE)
ROOT = os.path.dirname(TESTS)
for p in (ROOT, TESTS):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

import golden_cases  # noqa: E402
from helpers import digest  # noqa: E402


def main(names):
    path = os.path.join(HERE, "digests.json")
    digests = {}
    if os.path.exists(path):
        with open(path) as f:
            digests = json.load(f)
    for case in names:
        inputs, arrays, outs = getattr(golden_cases, case)()
        digests = {k: v for k, v in digests.items() if not k.startswith(case + "/")}
        for k, a in inputs.items():
            digests[f"{case}/input/{k}"] = digest(a)
        for k, a in outs.items():
            digests[f"{case}/{k}"] = digest(a)
        np.savez_compressed(os.path.join(HERE, case + ".npz"), **arrays)
        size = os.path.getsize(os.path.join(HERE, case + ".npz"))
        print(f"{case}: {len(arrays)} arrays ({size} B), {len(inputs) + len(outs)} digests")
    with open(path, "w") as f:
        json.dump(dict(sorted(digests.items())), f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main(sys.argv[1:] or golden_cases.CASES)
