"""The rank-set check across processes: four gloo ranks on the CPU, each
holding only its own rank file, reach the verdict validate_rank_set reaches
with all four files in one process -- pass for a consistent set, RankSet on
every rank for a set whose rank 3 diverges (a tensor name) or whose files are
in the wrong slots."""
import os
import pickle

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from glmaxx_b200 import rank_file as R
from tests.test_rank_file import family, to_product

WORLD = 4


def _worker(rank, port, paths, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=60))
    verdict = "ok"
    try:
        with R.NativeRankReader.open(paths[rank]) as rd:
            try:
                R.validate_rank_set_distributed(rd)
            except R.RankFileError as e:
                verdict = e.kind
    finally:
        dist.destroy_process_group()
    with open(os.path.join(out_dir, f"v{rank}.pkl"), "wb") as f:
        pickle.dump(verdict, f)


def _run(tmp_path, paths, port):
    mp.start_processes(_worker, args=(port, [str(p) for p in paths], str(tmp_path)),
                       nprocs=WORLD, join=True, start_method="spawn")
    out = []
    for r in range(WORLD):
        with open(tmp_path / f"v{r}.pkl", "rb") as f:
            out.append(pickle.load(f))
    return out


def _write(tmp_path, fam, tag):
    builders = [to_product(r, m, s, ident) for r, m, s, ident in fam]
    conv = R.RankFileBuilder.derive_conversion_uuid(builders)
    paths = []
    for b in builders:
        p = tmp_path / f"{tag}{b.rank}.g5n"
        b.write(p, conv)
        paths.append(p)
    return paths


@pytest.mark.parametrize("case", ["consistent", "divergent-name", "swapped"])
def test_rank_set_across_processes(tmp_path, case):
    fam = family("reader")
    if case == "divergent-name":
        from tests.test_rank_file import reader_specs
        r, m, _, ident = fam[3]
        fam[3] = (r, m, reader_specs(3, plain_name="model.test.divergent.weight"), ident)
    paths = _write(tmp_path, fam, case)
    if case == "swapped":
        paths = [paths[1], paths[0], paths[2], paths[3]]
    port = 29700 + ["consistent", "divergent-name", "swapped"].index(case)
    verdicts = _run(tmp_path, paths, port)
    # the same verdict as the single-process check, on every rank
    readers = [R.NativeRankReader.open(p) for p in paths]
    try:
        R.NativeRankReader.validate_rank_set(readers)
        want = "ok"
    except R.RankFileError as e:
        want = e.kind
    finally:
        for rd in readers:
            rd.close()
    assert verdicts == [want] * WORLD
    assert want == ("ok" if case == "consistent" else "RankSet")
