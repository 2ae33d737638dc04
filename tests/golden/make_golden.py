"""Extract the reference's golden vectors for the routed-MoE path into golden.json.

Run in a container where the reference checkout is mounted (its path is given on
the command line); the tests only read the committed golden.json, never the
reference itself.  Every value below is copied from the reference file:line
named beside it, read as text.

    python tests/golden/make_golden.py <reference-root>
"""
from __future__ import annotations

import json
import re
import sys
from pathlib import Path


def main(root: Path) -> None:
    fx = json.loads((root / "fixtures/sm120-fc1-matrix-proof-v1.json").read_text())
    actual = json.loads((root / "fixtures/nvfp4-actual-shape-v1.json").read_text())
    warp = json.loads((root / "fixtures/exl3-warp-staging-proof-v2.json").read_text())
    exl3_src = (root / "crates/glm-format/src/exl3.rs").read_text()
    fc1_src = (root / "crates/glm-reference/src/routed_fc1.rs").read_text()
    # exl3.rs:710-725 -- native-decode digest of the seeded fixture, as a byte list
    m = re.search(r"fn native_decode_has_stable_content_digest.*?\[(.*?)\]\s*\)", exl3_src, re.S)
    digest = bytes(int(b, 16) for b in re.findall(r"0x([0-9a-f]{2})", m.group(1)))
    # routed_fc1.rs:273-295 -- fixed-shape sequential / fixed-tree bit patterns
    bits = re.findall(r"to_bits\(\), (0x[0-9a-f_]+)\)", fc1_src)
    golden = {
        "source": "yatesdr/glmaxx fixtures and in-module tests (see make_golden.py)",
        "actual_shape": {  # fixtures/nvfp4-actual-shape-v1.json:1-29
            "n": actual["logical_shape"][0], "k": actual["logical_shape"][1],
            "packed_sha256": actual["packed_fixture_sha256"],
            "value_bytes": actual["packing"]["value_bytes"],
            "scale_bytes": actual["packing"]["scale_bytes"],
        },
        "matrix_proof": {  # fixtures/sm120-fc1-matrix-proof-v1.json
            "model_shape": fx["model_shape"],
            "row_buckets": fx["row_buckets"],
            "routing": fx["routing"],
            "numerical": fx["numerical"],
        },
        "fc1_fixed_shape": {  # crates/glm-reference/src/routed_fc1.rs:273-295
            "rows": 256, "n": 1024, "k": 6144, "row": 239, "column": 20,
            "sequential_bits": int(bits[0].replace("_", ""), 16),
            "fixed_tree_bits": int(bits[1].replace("_", ""), 16),
        },
        "fc2_toy": {  # crates/glm-reference/src/routed_fc2.rs:285-318
            "expected": [1.75, 3.5], "tolerance": [0.2, 0.4],
        },
        "finish_rank_order": {"expected": 116.0},  # routed_fc2.rs:364-376
        "exl3_native": {  # crates/glm-format/src/exl3.rs:667-725
            "k": 6144, "n": 512, "bits": 3, "seed": 0x0002C0260721,
            "sha256": digest.hex(),
        },
        "exl3_warp_proof": {  # fixtures/exl3-warp-staging-proof-v2.json:44-75, warp_proof.rs:67-68
            "rows": 8,
            "shapes": [
                {"family": s["projection_family"], "k": s["logical_k"], "n": s["logical_n"],
                 "seed": seed, "weight_sha256": s["scalar_weight_sha256"],
                 "projection_f16_sha256": s["scalar_projection_f16_sha256"]}
                for s, seed in zip(warp["shapes"], [0x3A4E2F157C91B608, 0xA2765CF811D049EB])
            ],
        },
        "scale_offset_closed_form": [  # crates/glm-format/tests/nvfp4_proof.rs:55-61
            [1, 0, 128, 64, 16], [32, 0, 128, 64, 4], [127, 3, 128, 64, 511],
            [128, 0, 256, 64, 512],
        ],
    }
    out = Path(__file__).resolve().parent / "golden.json"
    out.write_text(json.dumps(golden, indent=1) + "\n")
    print(f"wrote {out}")


if __name__ == "__main__":
    main(Path(sys.argv[1]))
