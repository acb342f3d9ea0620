"""Record the reference's ``patch_model`` decisions on the module zoo of ``patch_zoo.py``.

    python tests/golden/make_patch_golden.py --reference /path/to/TinKer

Imports the reference checkout (eb1386/TinKer), runs its ``tinker.patch_model`` on the CPU
over a fresh zoo for each flag set in ``patch_zoo.FLAG_SETS`` and writes, per flag set,
what sits at each path afterwards to ``patch_decisions.json`` beside this script.
"""

import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import patch_zoo  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TINKER_REFERENCE"),
                    help="path of the eb1386/TinKer checkout (or set TINKER_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference checkout with --reference PATH or the TINKER_REFERENCE variable")
    sys.path.insert(0, args.reference)
    import tinker
    out = {}
    for key, flags in patch_zoo.FLAG_SETS.items():
        model = tinker.patch_model(patch_zoo.zoo(), **flags)
        out[key] = patch_zoo.describe(model)
    with open(os.path.join(HERE, "patch_decisions.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print("wrote", os.path.join(HERE, "patch_decisions.json"))


if __name__ == "__main__":
    main()
