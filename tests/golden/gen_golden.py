"""Writes tests/golden/<case>.npz: the outputs of Trochilus's own code (oracle/_ref, built from the
reference sources by oracle/Makefile) for each case of cases.py, with a digest of the inputs so a test
can tell a changed generator from a changed result. Run in the development container:

    python tests/golden/gen_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.oracle import RefLib, make_desc  # noqa: E402
from tests.golden.cases import CASES, build_case, digest  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def main():
    ref = RefLib()
    pool = ref.pool(0)
    for c in CASES:
        lay, bias, normed, x = build_case(c)
        d, keep = make_desc(lay, c["H"], c["F"], c["k"], c["norm_topk"], c["router"], c["gate"], c["down"], bias)
        r = ref.moe_layer(d, normed, x, pool=pool)
        np.savez_compressed(os.path.join(OUT, c["name"] + ".npz"), digest=np.array(digest(lay, bias, normed, x)),
                            x=r["x"], logits=r["logits"], sel_id=r["sel_id"], sel_w=r["sel_w"], offsets=r["offsets"],
                            place=r["place"], ffn_out=r["ffn_out"], tier=np.array(ref.tier()),
                            q4_road=np.array(r["rc"]))
        print(c["name"], "road", r["rc"], "nan outputs", int(np.isnan(r["x"]).sum()), file=sys.stderr)
    ref.pool_destroy(pool)


if __name__ == "__main__":
    main()
