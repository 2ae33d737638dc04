"""Native rank-file (.g5n) reader and writer against the oracle restatement.

The fixtures restate the reference's own container and reader tests
(crates/glm-format/src/container.rs:1296-1665, native_reader.rs:1129-1547):
the 128x64 NVFP4 gate/up record, the layer-78 EXL3 projection, the padded
bf16 plain tensor, the three-tensor reader fixture.  Every file the product
writer makes must equal the oracle writer's bytes; every defect must give the
same error kind from the native reader, from the oracle reader and from the
reference (the kind its test asserts)."""
import ctypes
import hashlib
import os
import struct

import numpy as np
import pytest

import oracle as O
from oracle import rank_file as OR
from glmaxx_b200 import rank_file as R

KERNEL_ABI = b"glmaxx.sm120.nvfp4.routed_moe.v2"  # crates/glm-format/src/lib.rs:59
IDENT = tuple(hashlib.sha256(x).digest() for x in
              (b"config", b"tokenizer", b"template", b"policy", KERNEL_ABI))
READER_IDENT = tuple(bytes([i]) * 32 for i in (1, 2, 3, 4, 5))


# ------------------------------------------------------------------ fixtures
def container_input() -> np.ndarray:
    """(index % 31 - 15) / 7 in f32 over 128x64 (container.rs:1302-1305)."""
    i = np.arange(128 * 64, dtype=np.float32)
    return ((i % np.float32(31) - np.float32(15)) / np.float32(7)).reshape(128, 64)


def reader_nvfp4_input(rank: int) -> np.ndarray:
    """((index*17 + rank*3) % 127) / 31 - 2 over 129x65 (native_reader.rs:1201-1204)."""
    i = np.arange(129 * 65, dtype=np.int64)
    return (((i * 17 + rank * 3) % 127).astype(np.float32) / np.float32(31) -
            np.float32(2)).reshape(129, 65)


def exl3_parts(rank: int, projection: int = 1, layer: int = 78, k: int = 128, n: int = 128):
    """exl3_fixture (container.rs:1327-1337): trellis word i = i * 40503 mod 2^16."""
    words = (k // 16) * (n // 16) * 48
    trellis = (np.arange(words, dtype=np.uint32) * 40503 & 0xFFFF).astype(np.uint16)
    return dict(projection=projection, layer=layer, expert=0, rank=rank, k=k, n=n,
                trellis=trellis, suh=np.full(k, 0x3C00, np.uint16),
                svh=np.full(n, 0x3C00, np.uint16), marker=R.EXL3_MCG_MULTIPLIER)


def plain_bf16_bytes(rank: int) -> bytes:
    vals = [rank * 100 + 1, rank * 100 + 2, rank * 100 + 3, 0, rank * 100 + 4, rank * 100 + 5,
            rank * 100 + 6, 0]
    return struct.pack("<8H", *vals)


def spec(name, role, layer, expert, axis, flags, payload):
    return dict(name=name, role=role, layer=layer, expert=expert, axis=axis, flags=flags,
                payload=payload)


def to_product(rank: int, manifest: bytes, specs, ident) -> R.RankFileBuilder:
    """The same records as a product RankFileBuilder."""
    tensors = []
    for i, s in enumerate(specs):
        p = s["payload"]
        if p[0] == "plain":
            _, codec, ndim, ls, ps, data = p
            payload = R.PlainTensor({1: "bf16", 2: "fp16", 3: "fp32"}[codec], ndim, ls, ps, data)
        elif p[0] == "nvfp4":
            k = p[1]
            pn, pk = O.padded(k.n, k.k)
            payload = R.Nvfp4Tensor(k.n, k.k, pn, pk, k.global_scale, k.global_amax, k.values,
                                    k.scales, two_d=k.codec == "2d")
        else:
            _, proj, layer, expert, r, kk, nn, trellis, suh, svh, marker = p
            payload = R.Exl3Tensor(proj, layer, expert, r, kk, nn, trellis, suh, svh,
                                   mcg_marker=marker)
        tensors.append(R.TensorRecord(i, s["name"], s["role"], s["layer"], s["expert"], s["axis"],
                                      s["flags"], payload))
    return R.RankFileBuilder(rank, manifest, *ident, tensors=tensors)


def exl3_payload(e):
    return ("exl3", e["projection"], e["layer"], e["expert"], e["rank"], e["k"], e["n"],
            e["trellis"], e["suh"], e["svh"], e["marker"])


def container_specs(rank: int):
    return [spec("model.layers.3.mlp.experts.0.gate_up_proj.weight", 0x0501, 3, 0, 0, 0b1010,
                 ("nvfp4", O.pack(container_input(), "1d")))]


def exl3_specs(rank: int, projection: int = 1):
    return [spec("model.layers.78.mlp.experts.0.gate_proj.weight", 0x0501, 78, 0, 0, 0b1010,
                 exl3_payload(exl3_parts(rank, projection)))]


def plain_specs(rank: int, data=None):
    return [spec("model.layers.3.mlp.gate.e_score_correction_bias", 0x0302, 3, -1, -1, 1,
                 ("plain", 1, 2, (2, 3, 1, 1), (2, 4, 1, 1),
                  data if data is not None else bytes([1, 0, 2, 0, 3, 0, 0, 0, 4, 0, 5, 0, 6, 0,
                                                       0, 0])))]


def reader_specs(rank: int, exl3_projection: int = 1, plain_name="model.test.plain.weight"):
    return [spec(plain_name, 1, -1, -1, -1, 1,
                 ("plain", 1, 2, (2, 3, 1, 1), (2, 4, 1, 1), plain_bf16_bytes(rank))),
            spec("model.test.nvfp4.weight", 0x0501, 3, 0, 0, 0b1010,
                 ("nvfp4", O.pack(reader_nvfp4_input(rank), "1d"))),
            spec("model.test.exl3.weight", 0x0501, 78, 0, 0, 0b1010,
                 exl3_payload(exl3_parts(rank, exl3_projection)))]


def manifest(rank: int, schema: str) -> bytes:
    return ('{"rank":%d,"schema":"%s"}' % (rank, schema)).encode()


def family(kind: str, **kw):
    """Four ranks of one fixture family: (rank, manifest, specs, identities)."""
    out = []
    for r in range(4):
        if kind == "container":
            out.append((r, manifest(r, "test-v1"), container_specs(r), IDENT))
        elif kind == "exl3":
            out.append((r, manifest(r, "exl3-source-test-v1"), exl3_specs(r), IDENT))
        elif kind == "plain":
            out.append((r, manifest(r, "plain-test-v1"), plain_specs(r), IDENT))
        elif kind == "mixed":
            s = container_specs(r) + [spec("model.layers.78.mlp.experts.0.gate_proj.weight",
                                           0x0501, 78, 0, 0, 0b1010,
                                           exl3_payload(exl3_parts(r)))]
            out.append((r, manifest(r, "test-v1"), s, IDENT))
        elif kind == "exl3+nvfp4":
            s = exl3_specs(r) + [dict(container_specs(r)[0])]
            out.append((r, manifest(r, "exl3-source-test-v1"), s, IDENT))
        elif kind == "reader":
            out.append((r, manifest(r, "reader-test"), reader_specs(r, **kw), READER_IDENT))
    return out


def oracle_files(fam):
    conv = OR.conversion_uuid([(r, m, s) for r, m, s, _ in fam])
    return conv, [OR.build(r, m, s, conv, ident) for r, m, s, ident in fam]


def native_verdict(tmp_path, data: bytes, name="f.g5n"):
    """'ok' or the error kind: open, then verify."""
    path = tmp_path / name
    path.write_bytes(data)
    try:
        with R.NativeRankReader.open(path) as rd:
            rd.verify()
    except R.RankFileError as e:
        return e.kind
    return "ok"


def oracle_verdict(data: bytes):
    try:
        OR.Reader(data).verify()
    except OR.OracleRankError as e:
        return e.kind
    return "ok"


# ------------------------------------------------------------------ primitives
def test_hash_primitives():
    rng = np.random.default_rng(3)
    data = rng.integers(0, 256, 200_000, dtype=np.uint8).tobytes()
    for n in (0, 1, 55, 56, 63, 64, 65, 127, 128, 1000, 200_000):
        assert R.sha256(data[:n]) == hashlib.sha256(data[:n]).digest()
        assert R.crc32c(data[:n]) == O.crc32c(data[:n])
    R.sha256_force_portable(True)
    try:
        for n in (0, 63, 64, 65, 200_000):
            assert R.sha256(data[:n]) == hashlib.sha256(data[:n]).digest()
    finally:
        R.sha256_force_portable(False)
    assert R.crc32c(b"123456789") == 0xE3069283  # crc32c.rs standard check value


# ------------------------------------------------------------------ writer
@pytest.mark.parametrize("kind", ["container", "exl3", "plain", "mixed", "reader"])
def test_writer_bytes_equal_oracle_writer(kind):
    fam = family(kind)
    conv, files = oracle_files(fam)
    builders = [to_product(r, m, s, ident) for r, m, s, ident in fam]
    assert R.RankFileBuilder.derive_conversion_uuid(builders) == conv
    for b, f in zip(builders, files):
        assert b.build(conv) == f
        assert b.build(conv) == f  # deterministic (container.rs:1423-1440)


def test_writer_file_equals_build(tmp_path):
    fam = family("reader")
    b = to_product(*fam[1][:3], fam[1][3])
    conv = bytes(range(16))
    size = b.write(tmp_path / "w.g5n", conv)
    data = (tmp_path / "w.g5n").read_bytes()
    assert size == len(data) and data == b.build(conv)


def test_writer_rejections():
    bad = bytearray(plain_specs(0)[0]["payload"][5])
    bad[6] = 1  # a padding element (container.rs:1544-1549)
    with pytest.raises(R.RankFileError) as e:
        to_product(0, manifest(0, "plain-test-v1"),
                   plain_specs(0, data=bytes(bad)), IDENT).build(bytes(16))
    assert e.value.kind == "NonCanonicalLayout"
    specs = exl3_specs(0)
    p = list(specs[0]["payload"])
    p[10] ^= 1  # codebook marker (container.rs:1552-1563)
    specs[0]["payload"] = tuple(p)
    with pytest.raises(R.RankFileError) as e:
        to_product(0, manifest(0, "exl3-source-test-v1"), specs, IDENT).build(bytes(16))
    assert e.value.kind == "Exl3(CodebookMarker)"


# ------------------------------------------------------------------ reader
def test_four_rank_set_streams_once(tmp_path):
    """four_rank_images_stream_once_with_bounded_scratch (native_reader.rs:1296-1337)."""
    conv, files = oracle_files(family("reader"))
    readers = []
    for r, data in enumerate(files):
        (tmp_path / f"rank-{r}.g5n").write_bytes(data)
        readers.append(R.NativeRankReader.open(tmp_path / f"rank-{r}.g5n"))
    R.NativeRankReader.validate_rank_set(readers)
    OR.validate_rank_set([OR.Reader(f) for f in files])

    class Collect:
        def __init__(self):
            self.names, self.primary, self.aux, self.max_chunk = [], [], [], 0

        def begin_tensor(self, rank, index, name, descriptor):
            self.names.append(name)
            self.primary.append(b"")
            self.aux.append(b"")

        def primary_chunk(self, b):
            self.max_chunk = max(self.max_chunk, len(b))
            self.primary[-1] += b

        def aux_chunk(self, b):
            self.max_chunk = max(self.max_chunk, len(b))
            self.aux[-1] += b

        def finish_tensor(self):
            pass

    for rd, data in zip(readers, files):
        sink = Collect()
        proof = rd.verify_and_stream(sink)
        assert proof.tensor_count == 3 and bytes(proof.payload_sha256) == rd.payload_sha256
        assert proof.maximum_reader_scratch_bytes >= R.STREAM_CHUNK_BYTES
        assert sink.max_chunk <= R.STREAM_CHUNK_BYTES
        assert sink.names == ["model.test.plain.weight", "model.test.nvfp4.weight",
                              "model.test.exl3.weight"]
        assert len(sink.primary[0]) == 16 and sink.aux[0] == b""
        o = OR.Reader(data)
        o.verify()
        for i in range(3):
            assert (sink.primary[i], sink.aux[i]) == tuple(bytes(x) for x in o.planes(i))
        assert rd.conversion_uuid == conv and rd.tensor_name(2) == "model.test.exl3.weight"
        assert rd.tensor_codec_metadata(1) == bytes(o.b[o.d[1]["mo"]:o.d[1]["mo"] + 128])
    for rd in readers:
        rd.close()


def test_header_flags_and_descriptor_fields(tmp_path):
    for kind, flags in (("exl3", R.FLAG_EXL3), ("plain", R.FLAG_DIRECT_KERNEL),
                        ("mixed", R.FLAG_NVFP4 | R.FLAG_EXL3 | R.FLAG_HYBRID),
                        ("container", R.FLAG_DIRECT_KERNEL | R.FLAG_NVFP4)):
        _, files = oracle_files(family(kind))
        (tmp_path / f"{kind}.g5n").write_bytes(files[0])
        with R.NativeRankReader.open(tmp_path / f"{kind}.g5n") as rd:
            assert rd.header_flags == flags
            rd.verify()
            if kind == "exl3":
                d = rd.descriptors[0]
                assert (d.codec_id, d.logical_dtype, d.stored_dtype, d.quant_group_elements,
                        d.exl3_projection) == (0x0200, 2, 10, 0, 1)
            if kind == "plain":
                d = rd.descriptors[0]
                assert (d.codec_id, d.ndim, d.payload_bytes, d.aux_bytes,
                        d.codec_metadata_bytes) == (1, 2, 16, 0, 0)


def test_host_placement_bytes(tmp_path):
    """Placed planes land byte for byte where the placement says; the EXL3 aux
    plane splits into suh and svh; NVFP4 global scale from the metadata."""
    _, files = oracle_files(family("reader"))
    (tmp_path / "p.g5n").write_bytes(files[2])
    o = OR.Reader(files[2])
    with R.NativeRankReader.open(tmp_path / "p.g5n") as rd:
        plain = np.zeros(16, np.uint8)
        values = np.zeros(rd.descriptors[1].payload_bytes, np.uint8)
        scales = np.zeros(rd.descriptors[1].aux_bytes, np.uint8)
        gscale = np.zeros(1, np.float32)
        trellis = np.zeros(rd.descriptors[2].payload_bytes, np.uint8)
        suh, svh = np.zeros(128, np.uint16), np.zeros(128, np.uint16)
        placements = [(0, plain), (1, values, scales, gscale), (2, trellis, suh, svh)]
        with pytest.raises(R.RankFileError) as e:  # EXL3 source needs the explicit flag
            rd.load(placements, host=True)
        assert e.value.kind == "Argument"
        proof = rd.load(placements, host=True, exl3_source=True)
        assert plain.tobytes() == bytes(o.planes(0)[0])
        assert values.tobytes() == bytes(o.planes(1)[0])
        assert scales.tobytes() == bytes(o.planes(1)[1])
        assert gscale[0] == np.float32(o.codec_meta[1]["gs"])
        assert trellis.tobytes() == bytes(o.planes(2)[0])
        aux = bytes(o.planes(2)[1])
        assert suh.tobytes() == aux[4:260] and svh.tobytes() == aux[260:]
        assert proof.device_bytes == 16 + values.nbytes + scales.nbytes + 4 + trellis.nbytes + 512
        with pytest.raises(R.RankFileError) as e:  # one placement per tensor
            rd.load([(0, plain), (0, plain)], host=True)
        assert e.value.kind == "Argument"
        for short in ([(0, plain[:15])], [(1, values, scales[:-1], None)],
                      [(1, None, None, gscale.view(np.uint8)[:3])],
                      [(2, None, suh[:127], None)]):  # every destination holds its plane
            with pytest.raises(R.RankFileError) as e:
                rd.load(short, host=True, exl3_source=True)
            assert e.value.kind == "Argument"


def _descriptor_start(b):
    return struct.unpack_from("<Q", b, 56)[0]


def _rehash_plane(b, desc, which):
    """Update the descriptor digest of plane 'primary' or 'aux' after an edit."""
    off_f, len_f, dst = {"primary": (72, 80, 128), "aux": (88, 96, 160)}[which]
    o, n = struct.unpack_from("<QQ", b, desc + off_f)
    b[desc + dst:desc + dst + 32] = hashlib.sha256(bytes(b[o:o + n])).digest()


def _case(name):
    """One defect: (fixture family, edit(bytearray) -> bytearray, reference kind)."""
    def unknown_codec(b):  # container.rs:1566-1576
        struct.pack_into("<H", b, _descriptor_start(b) + 16, 0x7777)
        OR.resign_header(b)
        return b

    def flag_lie(b):  # container.rs:1578-1584
        struct.pack_into("<I", b, 20, R.FLAG_EXL3)
        OR.resign_header(b)
        return b

    def internal_padding(b):  # container.rs:1588-1609
        d = _descriptor_start(b)
        ao, ab = struct.unpack_from("<QQ", b, d + 88)
        assert b[ao + ab] == 0
        b[ao + ab] = 1
        OR.resign_header(b)
        return b

    def last_byte(b):  # container.rs:1612-1622 / native_reader.rs:1340-1368
        b[-1] ^= 1
        return b

    def metadata_lie(off):  # container.rs:1624-1643
        def edit(b):
            d = _descriptor_start(b)
            mo = struct.unpack_from("<Q", b, d + 104)[0]
            b[mo + off] ^= 0x02
            b[mo + 120:mo + 124] = bytes(4)
            struct.pack_into("<I", b, mo + 120, O.crc32c(bytes(b[mo:mo + 128])))
            b[d + 192:d + 224] = hashlib.sha256(bytes(b[mo:mo + 128])).digest()
            OR.resign_header(b)
            return b
        return edit

    def reserved_header(b):  # container.rs:1646-1656
        b[36] = 1
        b[416:420] = bytes(4)
        struct.pack_into("<I", b, 416, O.crc32c(bytes(b[:4096])))
        return b

    def trailing(b):  # container.rs:1658-1663
        return b + b"\0"

    def plain_padding(b):  # native_reader.rs:1389-1405
        d = _descriptor_start(b)
        po = struct.unpack_from("<Q", b, d + 72)[0]
        b[po + 6] = 1
        _rehash_plane(b, d, "primary")
        OR.resign_header(b)
        return b

    def nvfp4_value_padding(b):  # native_reader.rs:1407-1425
        d = _descriptor_start(b) + 256
        po = struct.unpack_from("<Q", b, d + 72)[0]
        b[po + 65 // 2] |= 0x10
        _rehash_plane(b, d, "primary")
        OR.resign_header(b)
        return b

    def nvfp4_zero_scale(b):  # native_reader.rs:1427-1443
        d = _descriptor_start(b) + 256
        ao = struct.unpack_from("<Q", b, d + 88)[0]
        assert b[ao] != 0
        b[ao] = 0
        _rehash_plane(b, d, "aux")
        OR.resign_header(b)
        return b

    def nvfp4_scale_nan(b):
        d = _descriptor_start(b) + 256
        ao = struct.unpack_from("<Q", b, d + 88)[0]
        b[ao] = 0x7F
        _rehash_plane(b, d, "aux")
        OR.resign_header(b)
        return b

    def exl3_marker(b):
        d = _descriptor_start(b) + 512
        ao = struct.unpack_from("<Q", b, d + 88)[0]
        b[ao] ^= 1
        _rehash_plane(b, d, "aux")
        OR.resign_header(b)
        return b

    def exl3_rotation(b):
        d = _descriptor_start(b) + 512
        ao = struct.unpack_from("<Q", b, d + 88)[0]
        struct.pack_into("<H", b, ao + 4 + 2 * 7, 0x7C00)  # suh[7] = +inf
        _rehash_plane(b, d, "aux")
        OR.resign_header(b)
        return b

    def header_crc(b):
        b[417] ^= 0xFF
        return b

    def magic(b):
        b[0] = ord("X")
        return b

    def truncated(b):
        return b[:4000]

    def rank(b):
        struct.pack_into("<I", b, 24, 5)
        OR.resign_header(b)
        return b

    def descriptor_reserved(b):
        b[_descriptor_start(b) + 26] = 1
        OR.resign_header(b)
        return b

    def name_control(b):
        so = struct.unpack_from("<Q", b, 72)[0]
        b[so + 2] = 0x07
        OR.resign_header(b)
        return b

    def file_uuid(b):
        b[380] ^= 1
        b[416:420] = bytes(4)
        struct.pack_into("<I", b, 416, O.crc32c(bytes(b[:4096])))
        return b

    def primary_digest(b):  # a flipped value byte, digests left alone
        d = _descriptor_start(b) + 256
        po = struct.unpack_from("<Q", b, d + 72)[0]
        b[po + 3] ^= 0x11
        return b

    def tensor_id(b):
        struct.pack_into("<I", b, _descriptor_start(b), 9)
        OR.resign_header(b)
        return b

    def region_gap(b):  # a nonzero byte between the manifest and the descriptors
        mo, mn = struct.unpack_from("<QQ", b, 40)
        b[mo + mn] = 1
        OR.resign_header(b)
        return b

    cases = {
        "unknown-codec": ("container", unknown_codec, "UnsupportedCodec"),
        "flag-lie": ("container", flag_lie, "HeaderFlags"),
        "internal-padding": ("exl3+nvfp4", internal_padding, "NonCanonicalLayout"),
        "last-byte": ("reader", last_byte, "TensorRegion"),
        "metadata-33": ("container", metadata_lie(33), "Nvfp4(UnsupportedMetadata)"),
        "metadata-52": ("container", metadata_lie(52), "Nvfp4(UnsupportedMetadata)"),
        "metadata-124": ("container", metadata_lie(124), "Nvfp4(UnsupportedMetadata)"),
        "reserved-header": ("container", reserved_header, "Header"),
        "trailing": ("reader", trailing, "Region"),
        "plain-padding": ("reader", plain_padding, "NonCanonicalLayout"),
        "nvfp4-value-padding": ("reader", nvfp4_value_padding, "Nvfp4(NonCanonicalPadding)"),
        "nvfp4-zero-scale": ("reader", nvfp4_zero_scale, "Nvfp4(ZeroScaleValue)"),
        "nvfp4-scale-nan": ("reader", nvfp4_scale_nan, "Nvfp4(ScaleEncoding)"),
        "exl3-marker": ("reader", exl3_marker, "Exl3(CodebookMarker)"),
        "exl3-rotation": ("reader", exl3_rotation, "Exl3(NonFiniteRotation)"),
        "header-crc": ("reader", header_crc, "HeaderCrc"),
        "magic": ("reader", magic, "Header"),
        "truncated": ("reader", truncated, "Truncated"),
        "rank": ("reader", rank, "Rank"),
        "descriptor-reserved": ("reader", descriptor_reserved, "Descriptor"),
        "name-control": ("reader", name_control, "StringTable"),
        "file-uuid": ("reader", file_uuid, "FileUuid"),
        "primary-digest": ("reader", primary_digest, "TensorRegion"),
        "tensor-id": ("reader", tensor_id, "TensorId"),
        "region-gap": ("reader", region_gap, "NonCanonicalLayout"),
    }
    return cases[name]


CASES = ["unknown-codec", "flag-lie", "internal-padding", "last-byte", "metadata-33",
         "metadata-52", "metadata-124", "reserved-header", "trailing", "plain-padding",
         "nvfp4-value-padding", "nvfp4-zero-scale", "nvfp4-scale-nan", "exl3-marker",
         "exl3-rotation", "header-crc", "magic", "truncated", "rank", "descriptor-reserved",
         "name-control", "file-uuid", "primary-digest", "tensor-id", "region-gap"]


@pytest.mark.parametrize("name", CASES)
def test_defect_verdicts(tmp_path, name):
    kind, edit, expected = _case(name)
    _, files = oracle_files(family(kind))
    assert native_verdict(tmp_path, files[0]) == "ok"
    bad = bytes(edit(bytearray(files[0])))
    assert oracle_verdict(bad) == expected
    assert native_verdict(tmp_path, bad, "bad.g5n") == expected


def test_nvfp4_2d_scale_sharing(tmp_path):
    """2-D codec: every row of a 16-row tile repeats the tile's scale
    (nvfp4.rs:446-455); a resigned file that breaks it is rejected."""
    x = container_input()
    specs = [spec("model.layers.3.mlp.experts.0.down_proj.weight", 0x0502, 3, 0, 1, 0b1100,
                  ("nvfp4", O.pack(x, "2d")))]
    conv = OR.conversion_uuid([(r, manifest(r, "t"), specs) for r in range(4)])
    data = bytearray(OR.build(0, manifest(0, "t"), specs, conv))
    assert native_verdict(tmp_path, bytes(data)) == "ok" and oracle_verdict(bytes(data)) == "ok"
    d = _descriptor_start(data)
    ao = struct.unpack_from("<Q", data, d + 88)[0]
    off = O.scale_offset(5, 0, 128, 64)  # row 5 of the first tile
    data[ao + off] = 0x3F if data[ao + off] != 0x3F else 0x3E
    _rehash_plane(data, d, "aux")
    OR.resign_header(data)
    assert oracle_verdict(bytes(data)) == "Nvfp4(ScaleSharing)"
    assert native_verdict(tmp_path, bytes(data), "bad.g5n") == "Nvfp4(ScaleSharing)"


def test_noncanonical_manifest(tmp_path):
    """native_reader.rs:1373-1387: reordered manifest keys, resigned."""
    _, files = oracle_files(family("reader"))
    b = bytearray(files[0])
    mo, mn = struct.unpack_from("<QQ", b, 40)
    repl = b'{"schema":"reader-test","rank":0}'
    assert len(repl) == mn
    b[mo:mo + mn] = repl
    OR.resign_header(b)
    assert native_verdict(tmp_path, bytes(b)) == "Manifest(NonCanonical)"


@pytest.mark.parametrize("divergence", ["name", "exl3-projection"])
def test_rank_set_divergence(tmp_path, divergence):
    """native_reader.rs:1445-1500: one rank's name or EXL3 projection differs."""
    fam = family("reader")
    r, m, s, ident = fam[3]
    s = reader_specs(3, plain_name="model.test.divergent.weight") if divergence == "name" else \
        reader_specs(3, exl3_projection=2)
    fam[3] = (r, m, s, ident)
    conv, files = oracle_files(fam)
    readers = []
    for i, data in enumerate(files):
        (tmp_path / f"d{i}.g5n").write_bytes(data)
        readers.append(R.NativeRankReader.open(tmp_path / f"d{i}.g5n"))
    with pytest.raises(R.RankFileError) as e:
        R.NativeRankReader.validate_rank_set(readers)
    assert e.value.kind == "RankSet"
    with pytest.raises(OR.OracleRankError) as e:
        OR.validate_rank_set([OR.Reader(f) for f in files])
    assert e.value.kind == "RankSet"
    # a rank file in the wrong slot
    swapped = [readers[1], readers[0], readers[2], readers[3]]
    with pytest.raises(R.RankFileError):
        R.NativeRankReader.validate_rank_set(swapped)
    for rd in readers:
        rd.close()


def test_unsafe_files_and_sink_failure(tmp_path):
    """native_reader.rs:1503-1546: hard links and symlinks are refused; a sink
    failure stops the stream."""
    _, files = oracle_files(family("reader"))
    path = tmp_path / "rank.g5n"
    path.write_bytes(files[0])
    link = tmp_path / "rank-link.g5n"
    os.link(path, link)
    with pytest.raises(R.RankFileError) as e:
        R.NativeRankReader.open(path)
    assert e.value.kind == "UnsafeFile"
    link.unlink()
    sym = tmp_path / "rank-sym.g5n"
    sym.symlink_to(path)
    with pytest.raises(R.RankFileError) as e:
        R.NativeRankReader.open(sym)
    assert e.value.kind == "UnsafeFile"

    class Failing:
        def begin_tensor(self, *a):
            pass

        def primary_chunk(self, b):
            raise RuntimeError("injected upload failure")

        def aux_chunk(self, b):
            pass

        def finish_tensor(self):
            pass

    with R.NativeRankReader.open(path) as rd:
        with pytest.raises(R.RankFileError) as e:
            rd.verify_and_stream(Failing())
        assert e.value.kind == "Sink" and e.value.message == "injected upload failure"
        rd.verify()  # the reader stays usable


def _big_family(experts=16, seed=5):
    """NVFP4 gate/up shards at the TP4 shape [1024, 6144] (3.1 MB values each),
    so planes straddle the 8 MiB stream chunks and several workers run."""
    rng = np.random.default_rng(seed)
    specs = []
    for e in range(experts):
        pn, pk = 1024, 6144
        values = rng.integers(0, 256, pn * pk // 2, dtype=np.uint8)
        scales = rng.integers(0x30, 0x40, pn * pk // 16, dtype=np.uint8)
        amax = np.float32(1.5 + e)
        packed = O.Packed(values, scales, np.float32(amax / np.float32(2688.0)), amax, pn, pk, "1d")
        specs.append(spec(f"model.layers.3.mlp.experts.{e}.gate_up_proj.weight", 0x0501, 3, e, 0,
                          0b1010, ("nvfp4", packed)))
    return specs


def test_multichunk_stream_and_placement(tmp_path):
    specs = _big_family()
    conv = OR.conversion_uuid([(r, manifest(r, "big"), specs) for r in range(4)])
    data = OR.build(0, manifest(0, "big"), specs, conv)
    assert len(data) > 6 * R.STREAM_CHUNK_BYTES  # more chunks than staging slots: slots reused
    product = to_product(0, manifest(0, "big"), specs, (bytes(32),) * 5)
    assert product.build(conv) == data
    path = tmp_path / "big.g5n"
    path.write_bytes(data)
    o = OR.Reader(data)
    with R.NativeRankReader.open(path) as rd:
        bufs = [(np.zeros(d.payload_bytes, np.uint8), np.zeros(d.aux_bytes, np.uint8))
                for d in rd.descriptors]
        proof = rd.load([(i, v, s, None) for i, (v, s) in enumerate(bufs)], host=True)
        assert proof.stream_chunks == -(-rd.file_payload_bytes() // R.STREAM_CHUNK_BYTES)
        for i, (v, s) in enumerate(bufs):
            assert v.tobytes() == bytes(o.planes(i)[0]) and s.tobytes() == bytes(o.planes(i)[1])
    # a flipped byte in the plane that straddles the first chunk boundary
    bad = bytearray(data)
    pay = struct.unpack_from("<Q", bad, 104)[0]
    bad[pay + R.STREAM_CHUNK_BYTES + 5] ^= 0x40
    assert oracle_verdict(bytes(bad)) == "TensorRegion"
    assert native_verdict(tmp_path, bytes(bad), "bad.g5n") == "TensorRegion"


def test_error_names_cover_header():
    text = (R.abi.LIB_PATH.parent.parent / "include" / "glmaxx_rank_file.h").read_text()
    import re
    codes = [int(v) for v in re.findall(r"GLMAXX_RANK_ERR_\w+ = (-\d+)", text)]
    assert len(codes) > 40
    for c in codes:
        assert R.error_name(c) not in ("Unknown", "Ok")
    assert len({R.error_name(c) for c in codes}) == len(codes)


def test_rank_file_abi_exports_and_layouts():
    """Every function include/glmaxx_rank_file.h declares is exported and bound;
    the ctypes mirrors have the C struct sizes (static_asserts in rank_file.cpp)."""
    import re
    text = (R.abi.LIB_PATH.parent.parent / "include" / "glmaxx_rank_file.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = sorted(set(re.findall(r"\b(glmaxx_[a-z0-9_]+)\s*\(", text)))
    assert len(names) == 15
    lib = R._load()
    for n in names:
        fn = getattr(lib, n)
        assert fn.argtypes is not None or n == "glmaxx_sha256_accelerated", n
    assert ctypes.sizeof(R.RankFileInfo) == 328
    assert ctypes.sizeof(R.TensorInfo) == 136
    assert ctypes.sizeof(R.Placement) == 56
    assert ctypes.sizeof(R.PayloadProof) == 88
    assert ctypes.sizeof(R._Sink) == 40


def _resign_all(b: bytearray) -> None:
    """Recompute every digest after an edit: each descriptor's plane and
    metadata digests, the metadata region digest, then the header."""
    d0, n = struct.unpack_from("<Q", b, 56)[0], struct.unpack_from("<I", b, 32)[0]
    for i in range(n):
        d = d0 + 256 * i
        try:
            for which in ("primary", "aux"):
                _rehash_plane(b, d, which)
            mo, mb = struct.unpack_from("<QQ", b, d + 104)
            b[d + 192:d + 224] = hashlib.sha256(bytes(b[mo:mo + mb])).digest()
        except struct.error:
            return
    OR.resign_header(b)


@pytest.mark.parametrize("resign", [False, True])
def test_fuzzed_files_same_verdict(tmp_path, resign):
    """Seeded single-byte edits anywhere in the reader fixture (control regions,
    descriptors, metadata, planes, padding): the native reader and the oracle
    reach the same verdict on every file."""
    _, files = oracle_files(family("reader"))
    base = files[0]
    rng = np.random.default_rng(1234 + resign)
    seen = {}
    for trial in range(160):
        b = bytearray(base)
        pos = int(rng.integers(0, len(b)))
        b[pos] ^= int(rng.integers(1, 256))
        if resign and pos >= 4096:
            try:
                _resign_all(b)
            except Exception:  # noqa: BLE001 -- an edited offset may point anywhere
                pass
        want = oracle_verdict(bytes(b))
        got = native_verdict(tmp_path, bytes(b), f"fuzz{trial}.g5n")
        assert got == want, (trial, pos, got, want)
        seen[want] = seen.get(want, 0) + 1
    assert len(seen) >= (4 if resign else 3), seen


@pytest.mark.parametrize("order", ["scale-encoding-first", "zero-scale-first"])
def test_earliest_tensor_error_wins_across_workers(tmp_path, order):
    """Two resigned defects in different tensors of a multi-chunk file (handled
    by different plane workers): the reader reports the earlier tensor's error,
    as the reference's in-order stream does, whichever worker finds its own
    defect first."""
    specs = _big_family()
    conv = OR.conversion_uuid([(r, manifest(r, "big"), specs) for r in range(4)])
    b = bytearray(OR.build(0, manifest(0, "big"), specs, conv))
    d0 = _descriptor_start(b)
    early, late = (3, 11)
    kinds = {"nan": "Nvfp4(ScaleEncoding)", "zero": "Nvfp4(ZeroScaleValue)"}
    first, second = ("nan", "zero") if order == "scale-encoding-first" else ("zero", "nan")
    for t, kind in ((early, first), (late, second)):
        d = d0 + 256 * t
        ao = struct.unpack_from("<Q", b, d + 88)[0]
        b[ao + 4096] = 0x7F if kind == "nan" else 0
        _rehash_plane(b, d, "aux")
    OR.resign_header(b)
    want = kinds[first]
    assert oracle_verdict(bytes(b)) == want
    assert native_verdict(tmp_path, bytes(b), "two.g5n") == want


def test_changed_file_and_concurrent_verifies(tmp_path):
    """ensure_unchanged (native_reader.rs:590-604): a file whose timestamps
    change after open is refused ("Changed"); two threads verifying through one
    handle take turns on its staging and both succeed."""
    import threading
    _, files = oracle_files(family("reader"))
    path = tmp_path / "r.g5n"
    path.write_bytes(files[0])
    with R.NativeRankReader.open(path) as rd:
        results = []

        def run():
            try:
                results.append(bytes(rd.verify().payload_sha256))
            except R.RankFileError as e:  # pragma: no cover - reported below
                results.append(e.kind)
        threads = [threading.Thread(target=run) for _ in range(2)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        assert results == [rd.payload_sha256] * 2
        st = os.stat(path)
        os.utime(path, ns=(st.st_atime_ns, st.st_mtime_ns + 1_000_000_000))
        with pytest.raises(R.RankFileError) as e:
            rd.verify()
        assert e.value.kind == "Changed"
