"""Record the reference's per-layer source schedules for every path topology.

Run from the repository root with the reference checkout available::

    python tests/golden/make_topology_table.py --reference <path to the reference checkout>

It imports ``BiAttn.topology`` from the reference and writes
``tests/golden/topology_table.json``: for every name in its
``PATH_TOPOLOGIES``, layers 1..22 and total_layers in (3, 12, 20), the tuple
``topology_offsets(layer, topology=name, total_layers=total)`` returns, or
null where that tuple has more than 64 offsets (``h3`` grows as 2**(l-1)).
The tests read only the JSON file.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

LAYERS = range(1, 23)
TOTALS = (3, 12, 20)


def _capped(offsets):
    return list(offsets) if len(offsets) <= 64 else None


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True)
    parser.add_argument("--out", default=os.path.join(os.path.dirname(__file__), "topology_table.json"))
    args = parser.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    from BiAttn import topology  # noqa: E402  (the reference's own module)

    table = {"topologies": list(topology.PATH_TOPOLOGIES), "layers": list(LAYERS), "totals": list(TOTALS),
             "offsets": {}}
    for name in topology.PATH_TOPOLOGIES:
        table["offsets"][name] = {
            str(total): [_capped(topology.topology_offsets(layer, topology=name, total_layers=total))
                         for layer in LAYERS]
            for total in TOTALS
        }
    with open(args.out, "w") as handle:
        json.dump(table, handle, separators=(",", ":"))
    print(f"wrote {args.out}: {len(table['topologies'])} topologies")


if __name__ == "__main__":
    main()
