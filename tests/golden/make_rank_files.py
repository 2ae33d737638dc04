"""Generate the committed rank-file fixtures tests/golden/rank_reader_rank{0..3}.g5n
and rank_files.json (per-file SHA-256, conversion UUID) with the oracle writer
(oracle/rank_file.py, the restatement of the reference's RankFileBuilder).

    python tests/golden/make_rank_files.py

The records are the reader test fixture of the reference
(crates/glm-format/src/native_reader.rs:1189-1268): per rank a padded bf16
plain tensor, a 129x65 NVFP4 tensor and a layer-78 128x128 EXL3 projection.
"""
import hashlib
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import rank_file as OR  # noqa: E402
from tests.test_rank_file import family  # noqa: E402


def main():
    fam = family("reader")
    conv = OR.conversion_uuid([(r, m, s) for r, m, s, _ in fam])
    files = {}
    for r, m, s, ident in fam:
        data = OR.build(r, m, s, conv, ident)
        name = f"rank_reader_rank{r}.g5n"
        (HERE / name).write_bytes(data)
        files[name] = hashlib.sha256(data).hexdigest()
    (HERE / "rank_files.json").write_text(json.dumps(
        {"conversion_uuid": conv.hex(), "files": files}, indent=1) + "\n")
    print(json.dumps(files, indent=1))


if __name__ == "__main__":
    main()
