"""Fixtures for the descriptor-emitter test, from the reference's fusion lit inputs.

    python tests/golden/make_emitter_golden.py /path/to/reference

Parses the fp-dialect functions of the reference's lit tests for the two fusion
passes (test/fusion/{fuse_chains,fuse_attention,dedupe_mul,two_softmax,
no_fuse_head_dim}.mlir) with the planner twin's parser, and writes next to this
script:

* ``emitter_inputs.mlir`` -- the same functions re-printed by the planner's
  printer (so the test needs no reference checkout);
* ``emitter_plans.json`` -- per function, the plan the twin compiles with both
  fusion passes on: steps, launch attrs and the ``attrs["desc"]`` descriptors
  that integration/PlanEmitter.descriptors.patch must emit for the same input.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from fusionpass_b200 import planner  # noqa: E402

LIT = ["fuse_chains.mlir", "fuse_attention.mlir", "dedupe_mul.mlir", "two_softmax.mlir", "no_fuse_head_dim.mlir"]


def main(argv) -> int:
    if len(argv) < 2:
        print("usage: python tests/golden/make_emitter_golden.py /path/to/reference", file=sys.stderr)
        return 2
    ref = Path(argv[1])
    texts, plans = [], {}
    for name in LIT:
        funcs = planner.parse_fp_mlir((ref / "test" / "fusion" / name).read_text())
        for fn, g in funcs.items():
            key = f"{Path(name).stem}.{fn}"
            texts.append(f"// {key}\n" + planner.to_mlir(g, key.replace(".", "__")))
            plan, _ = planner.compile_graph(planner.parse_fp_mlir(texts[-1])[key.replace(".", "__")], fuse=True)
            plans[key] = plan
    (HERE / "emitter_inputs.mlir").write_text("\n".join(texts))
    (HERE / "emitter_plans.json").write_text(json.dumps(plans, indent=1, sort_keys=True) + "\n")
    print(f"{len(plans)} functions")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
