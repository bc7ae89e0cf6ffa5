"""Record the reference's outcome (exception type and message) for every case
of ``contract_cases.error_cases`` into ``contract_errors.json``, by running
the REFERENCE implementation on CPU.

    python tests/golden/make_contract_golden.py --reference <reference checkout>

(or set TC_REFERENCE_ROOT).  The reference is imported through the same
symlink shim as ``make_golden.py``; nothing is copied.
"""

import argparse
import json
import os
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import contract_cases as CC  # noqa: E402
from make_golden import import_reference  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TC_REFERENCE_ROOT"),
                    help="reference checkout (default: $TC_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or TC_REFERENCE_ROOT")
    rs, ref = import_reference(args.reference)
    api = types.SimpleNamespace(**{n: getattr(ref, n) for n in ref.__all__})
    api.RangeSpec = rs.RangeSpec
    out = []
    for label, fn in CC.error_cases(api, "cpu"):
        etype, msg = CC.run_case(fn)
        out.append(dict(label=label, type=etype, message=msg))
        print(f"{label:45s} {etype}: {msg}")
    with open(os.path.join(HERE, "contract_errors.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
