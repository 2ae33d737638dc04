"""Committed rank-file fixtures (tests/golden/rank_reader_rank{0..3}.g5n, made
by tests/golden/make_rank_files.py with the oracle writer): the product writer
reproduces their bytes, the native reader and the oracle accept them, and the
four form a valid rank set -- fixed bytes, so the writer and the reader cannot
drift together."""
import hashlib
import json
from pathlib import Path

from oracle import rank_file as OR
from glmaxx_b200 import rank_file as R
from tests.test_rank_file import family, to_product

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_committed_rank_files():
    meta = json.loads((GOLDEN / "rank_files.json").read_text())
    conv = bytes.fromhex(meta["conversion_uuid"])
    fam = family("reader")
    builders = [to_product(r, m, s, ident) for r, m, s, ident in fam]
    assert R.RankFileBuilder.derive_conversion_uuid(builders) == conv
    readers = []
    for r, b in enumerate(builders):
        name = f"rank_reader_rank{r}.g5n"
        data = (GOLDEN / name).read_bytes()
        assert hashlib.sha256(data).hexdigest() == meta["files"][name]
        assert b.build(conv) == data
        OR.Reader(data).verify()
        rd = R.NativeRankReader.open(GOLDEN / name)
        proof = rd.verify()
        assert bytes(proof.payload_sha256) == rd.payload_sha256 and rd.conversion_uuid == conv
        readers.append(rd)
    R.NativeRankReader.validate_rank_set(readers)
    for rd in readers:
        rd.close()
