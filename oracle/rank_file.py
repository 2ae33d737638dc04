"""CPU restatement of the GLM-5.2 rank-file container -- TEST INFRASTRUCTURE ONLY.

Pure Python + numpy restatement of the reference's container writer and
native reader, used by ``tests/`` to check the product's writer
(``glmaxx_b200.rank_file.RankFileBuilder``) byte for byte and the product's C++
reader verdict for verdict.  It follows:

  writer  crates/glm-format/src/container.rs:236-470 (RankFileBuilder::prepare/build),
          :1037-1110 (encode_rank_header), :1116-1180 (EncodedTensor::from_record)
  open    crates/glm-format/src/native_reader.rs:119-335, :724-858 (validate_descriptors)
  verify  native_reader.rs:378-537 (verify_and_stream: per tensor, padding, primary
          plane validators and digest, padding, aux validators and digest, codec
          finish; whole-payload digest last)
  codecs  nvfp4.rs:84-160 (metadata), :309-464 (Nvfp4PlaneValidator);
          exl3.rs:72-157 (metadata), :229-340 (from_container_planes / validate)
  set     native_reader.rs:543-588 (validate_rank_set)

Errors raise ``OracleRankError(kind)`` with the reference variant name.
"""
from __future__ import annotations

import hashlib
import struct

import numpy as np

from . import crc32c

LAYOUT_SOURCE_SHA256 = bytes([
    0x59, 0x8e, 0x05, 0x4b, 0xef, 0x21, 0xed, 0xf9, 0x4b, 0x1f, 0xd6, 0xbb, 0x14, 0x47, 0xcf, 0xa9,
    0xcf, 0xcf, 0x5a, 0x59, 0x07, 0xab, 0x37, 0x01, 0x28, 0x10, 0x24, 0x48, 0xdb, 0xb6, 0xd5, 0x30])
QUANT_POLICY_SHA256 = bytes([
    0xcd, 0x90, 0x95, 0x79, 0x33, 0x44, 0x05, 0xec, 0xd4, 0xcd, 0x8d, 0x9a, 0x6c, 0x2d, 0xfc, 0xba,
    0x7f, 0x01, 0x24, 0xc4, 0xc4, 0xba, 0x92, 0xbc, 0x40, 0xc9, 0x76, 0xd5, 0x74, 0xbe, 0x05, 0xa3])
MCG = 0xCBAC1FED
PLAIN = {1: 2, 2: 2, 3: 4}  # codec -> element bytes
NVFP4 = (0x0100, 0x0101)
EXL3 = 0x0200


class OracleRankError(Exception):
    def __init__(self, kind: str):
        super().__init__(kind)
        self.kind = kind


def _fail(kind: str):
    raise OracleRankError(kind)


def _u16(b, o):
    return struct.unpack_from("<H", b, o)[0]


def _u32(b, o):
    return struct.unpack_from("<I", b, o)[0]


def _u64(b, o):
    return struct.unpack_from("<Q", b, o)[0]


def _sha(b) -> bytes:
    return hashlib.sha256(bytes(b)).digest()


def _align(v, a):
    return (v + a - 1) // a * a


# ----------------------------------------------------------------- metadata
def nvfp4_metadata(codec2d, ln, lk, pn, pk, gscale, gamax, vbytes, sbytes) -> bytes:
    """Nvfp4Metadata::encode (nvfp4.rs:40-78)."""
    b = bytearray(128)
    struct.pack_into("<HH", b, 0, 0, 1)
    struct.pack_into("<H", b, 4, 0x0101 if codec2d else 0x0100)
    b[6] = 2 if codec2d else 1
    b[7] = 1
    struct.pack_into("<IIII", b, 8, ln, lk, pn, pk)
    struct.pack_into("<HHHH", b, 24, 16, 16 if codec2d else 1, 0x1201, 0x1201)
    b[32:36] = bytes([1, 1, 1, 1])
    struct.pack_into("<ffII", b, 36, gscale, gamax, vbytes, sbytes)
    b[56:88] = LAYOUT_SOURCE_SHA256
    b[88:120] = QUANT_POLICY_SHA256
    struct.pack_into("<I", b, 120, crc32c(bytes(b)))
    return bytes(b)


def _nvfp4_validate(m):
    ln, lk, pn, pk = m["ln"], m["lk"], m["pn"], m["pk"]
    gs, ga = np.float32(m["gs"]), np.float32(m["ga"])
    if ln == 0 or lk == 0 or pn < ln or pk < lk or pn % 128 or pk % 64 or not np.isfinite(gs) or \
            gs <= 0 or not np.isfinite(ga) or np.signbit(ga):
        _fail("Nvfp4(InvalidShapeOrScale)")
    expected = np.float32(1.0) if ga == 0 else np.float32(ga / np.float32(2688.0))
    if gs.view(np.uint32) != expected.view(np.uint32):
        _fail("Nvfp4(InvalidShapeOrScale)")
    if m["vb"] != pn * pk // 2 or m["sb"] != pn * pk // 16:
        _fail("Nvfp4(ByteAccounting)")


def nvfp4_decode(b: bytes) -> dict:
    """Nvfp4Metadata::decode (nvfp4.rs:84-126)."""
    if len(b) != 128:
        _fail("Nvfp4(MetadataLength)")
    chk = bytearray(b)
    chk[120:124] = bytes(4)
    if crc32c(bytes(chk)) != _u32(b, 120):
        _fail("Nvfp4(MetadataCrc)")
    if _u16(b, 0) != 0 or _u16(b, 2) != 1 or b[7] != 1 or _u16(b, 24) != 16 or \
            _u16(b, 28) != 0x1201 or _u16(b, 30) != 0x1201 or bytes(b[32:36]) != b"\x01" * 4 or \
            bytes(b[52:56]) != bytes(4) or bytes(b[56:88]) != LAYOUT_SOURCE_SHA256 or \
            bytes(b[88:120]) != QUANT_POLICY_SHA256 or bytes(b[124:128]) != bytes(4):
        _fail("Nvfp4(UnsupportedMetadata)")
    c = _u16(b, 4)
    if c == 0x0100 and b[6] == 1 and _u16(b, 26) == 1:
        two_d = False
    elif c == 0x0101 and b[6] == 2 and _u16(b, 26) == 16:
        two_d = True
    else:
        _fail("Nvfp4(UnsupportedMetadata)")
    m = dict(two_d=two_d, ln=_u32(b, 8), lk=_u32(b, 12), pn=_u32(b, 16), pk=_u32(b, 20),
             gs=struct.unpack_from("<f", b, 36)[0], ga=struct.unpack_from("<f", b, 40)[0],
             vb=_u32(b, 44), sb=_u32(b, 48))
    _nvfp4_validate(m)
    return m


def _scale_offsets(pn, pk):
    """scale_offset(row, group) for all (row, group), row-major (nvfp4.rs:493-521)."""
    n = np.arange(pn, dtype=np.int64)[:, None]
    g = np.arange(pk // 16, dtype=np.int64)[None, :]
    return (512 * ((n // 128) * (pk // 64) + g // 4) + 16 * (n % 32) + 4 * ((n % 128) // 32) +
            g % 4)


def nvfp4_validate_planes(m, values: bytes, scales: bytes):
    """Nvfp4PlaneValidator value_chunk / scale_chunk / finish (nvfp4.rs:333-464)."""
    pn, pk, ln, lk = m["pn"], m["pk"], m["ln"], m["lk"]
    v = np.frombuffer(values, np.uint8).reshape(pn, pk // 16, 8)
    codes = np.stack([v & 15, v >> 4], axis=-1).reshape(pn, pk // 16, 16)
    row = np.arange(pn)[:, None]
    start = np.arange(pk // 16)[None, :] * 16
    outside = (row >= ln) | (start >= lk)
    lane_pad = (np.arange(16)[None, None, :] + start[:, :, None]) >= lk
    if np.any(codes[outside]) or np.any(codes[~outside[:, :, None].repeat(16, 2) & lane_pad]):
        _fail("Nvfp4(NonCanonicalPadding)")
    s = np.frombuffer(scales, np.uint8)
    if np.any((s & 0x80) != 0) or np.any(s == 0x7F):
        _fail("Nvfp4(ScaleEncoding)")
    off = _scale_offsets(pn, pk)
    sc = s[off]
    nonzero = np.any(v != 0, axis=-1)
    zero_fail = (sc == 0) & nonzero
    dom_row = (row // 16) * 16 < ln if m["two_d"] else row < ln
    domain = (start < lk) & dom_row
    pad_fail = ~domain & (sc != 0)
    share_fail = np.zeros_like(zero_fail)
    if m["two_d"]:
        share_fail = sc != sc[(np.arange(pn) // 16) * 16][:, :]
    first = np.flatnonzero((zero_fail | pad_fail | share_fail).reshape(-1))
    if first.size:
        i = first[0]
        if zero_fail.reshape(-1)[i]:
            _fail("Nvfp4(ZeroScaleValue)")
        if pad_fail.reshape(-1)[i]:
            _fail("Nvfp4(NonCanonicalPadding)")
        _fail("Nvfp4(ScaleSharing)")


def exl3_metadata(projection, layer, expert, rank, bits, k, n) -> bytes:
    """Exl3Metadata::encode (exl3.rs:104-122)."""
    b = bytearray(96)
    b[0:8] = b"GLX3TR3\x00"
    struct.pack_into("<HH", b, 8, 1, 1)
    b[12], b[13], b[14] = projection, bits, rank
    struct.pack_into("<HHIII", b, 16, layer, expert, k, n, MCG)
    struct.pack_into("<QQ", b, 32, (k // 16) * (n // 16) * 16 * bits, k + n)
    struct.pack_into("<I", b, 88, crc32c(bytes(b)))
    return bytes(b)


def exl3_decode(b: bytes) -> dict:
    """Exl3Metadata::decode + validate (exl3.rs:72-157)."""
    if len(b) != 96:
        _fail("Exl3(MetadataLength)")
    chk = bytearray(b)
    chk[88:92] = bytes(4)
    if crc32c(bytes(chk)) != _u32(b, 88):
        _fail("Exl3(MetadataCrc)")
    if bytes(b[:8]) != b"GLX3TR3\x00" or _u16(b, 8) != 1 or _u16(b, 10) != 1 or \
            _u32(b, 28) != MCG or b[15] != 0 or any(b[48:88]) or any(b[92:96]) or \
            b[12] not in (1, 2, 3):
        _fail("Exl3(UnsupportedContract)")
    m = dict(projection=b[12], bits=b[13], rank=b[14], layer=_u16(b, 16), expert=_u16(b, 18),
             k=_u32(b, 20), n=_u32(b, 24), trellis=_u64(b, 32), rotation=_u64(b, 40))
    k, n = m["k"], m["n"]
    if not 3 <= m["layer"] <= 78 or m["expert"] >= 256 or m["rank"] >= 4 or m["bits"] != 3 or \
            k == 0 or n == 0 or k % 128 or n % 128:
        _fail("Exl3(UnsupportedContract)")
    if m["trellis"] != (k // 16) * (n // 16) * 48 or m["rotation"] != k + n:
        _fail("Exl3(ByteAccounting)")
    if m["layer"] <= 77 and (k, n) != ((6144, 512) if m["projection"] in (1, 2) else (512, 6144)):
        _fail("Exl3(UnsupportedContract)")
    return m


# ----------------------------------------------------------------- writer
def encode_record(rec: dict, rank: int) -> dict:
    """EncodedTensor::from_record (container.rs:1116-1180).  rec["payload"] is
    ("plain", codec, ndim, logical4, padded4, bytes), ("nvfp4", oracle.Packed)
    or ("exl3", projection, layer, expert, rank, k, n, trellis_u16, suh_u16, svh_u16, marker)."""
    kind = rec["payload"][0]
    if kind == "plain":
        _, codec, ndim, lshape, pshape, data = rec["payload"]
        return dict(codec=codec, ld=codec, sd=codec, lshape=lshape, pshape=pshape, group=0,
                    ndim=ndim, aux_flag=0, meta=b"", primary=bytes(data), aux=b"")
    if kind == "nvfp4":
        p = rec["payload"][1]
        pn, pk = (p.n + 127) // 128 * 128, (p.k + 63) // 64 * 64
        return dict(codec=0x0101 if p.codec == "2d" else 0x0100, ld=1, sd=6,
                    lshape=(p.n, p.k, 1, 1), pshape=(pn, pk, 1, 1), group=16, ndim=2,
                    aux_flag=0x80, meta=p.metadata(), primary=p.values.tobytes(),
                    aux=p.scales.tobytes())
    _, proj, layer, expert, r, k, n, trellis, suh, svh, marker = rec["payload"]
    aux = struct.pack("<I", marker) + np.asarray(suh, "<u2").tobytes() + \
        np.asarray(svh, "<u2").tobytes()
    return dict(codec=EXL3, ld=2, sd=10, lshape=(n, k, 1, 1), pshape=(n, k, 1, 1), group=0,
                ndim=2, aux_flag=0x80, meta=exl3_metadata(proj, layer, expert, r, 3, k, n),
                primary=np.asarray(trellis, "<u2").tobytes(), aux=aux)


def _prepare(rank, manifest, records):
    man_off = 4096
    desc_off = _align(man_off + len(manifest), 4096)
    str_off = _align(desc_off + 256 * len(records), 4096)
    strings = b"".join(r["name"].encode() for r in records)
    meta_off = _align(str_off + len(strings), 4096)
    enc = [encode_record(r, rank) for r in records]
    metadata = b"".join(e["meta"] for e in enc)
    pay_off = _align(meta_off + len(metadata), 4096)
    payload, descs, name_cur, meta_cur = bytearray(), bytearray(), 0, 0
    for i, (r, e) in enumerate(zip(records, enc)):
        payload += bytes(_align(len(payload), 256) - len(payload))
        v_local = len(payload)
        payload += e["primary"]
        payload += bytes(_align(len(payload), 256) - len(payload))
        s_local = len(payload)
        payload += e["aux"]
        d = bytearray(256)
        nb = len(r["name"].encode())
        struct.pack_into("<IIHHhhHHHbBB", d, 0, i, name_cur, nb, r["role"], r["layer"],
                         r["expert"], e["codec"], e["ld"], e["sd"], r["axis"], e["ndim"],
                         r["flags"] | e["aux_flag"])
        struct.pack_into("<8I", d, 28, *e["lshape"], *e["pshape"])
        elements = int(np.prod(e["lshape"][:e["ndim"]], dtype=np.uint64))
        struct.pack_into("<7QII", d, 64, elements, pay_off + v_local, len(e["primary"]),
                         pay_off + s_local, len(e["aux"]), meta_off + meta_cur, len(e["meta"]),
                         256, e["group"])
        d[128:160] = _sha(e["primary"])
        d[160:192] = _sha(e["aux"])
        d[192:224] = _sha(e["meta"])
        descs += d
        name_cur += nb
        meta_cur += len(e["meta"])
    codecs = [e["codec"] for e in enc]
    return dict(man_off=man_off, desc_off=desc_off, str_off=str_off, meta_off=meta_off,
                pay_off=pay_off, descs=bytes(descs), strings=strings, metadata=metadata,
                payload=bytes(payload), flags=header_flags(codecs))


def header_flags(codecs) -> int:
    """derive_header_flags (container.rs:816-844)."""
    plain = any(c in PLAIN for c in codecs)
    nv = any(c in NVFP4 for c in codecs)
    ex = any(c == EXL3 for c in codecs)
    for c in codecs:
        if c not in PLAIN and c not in NVFP4 and c != EXL3:
            _fail("UnsupportedCodec")
    return (1 if (plain or nv) and not ex else 0) | (2 if nv else 0) | (4 if ex else 0) | \
        (16 if nv and ex else 0)


def conversion_uuid(ranks) -> bytes:
    """ranks: four (rank, manifest, records) triples (format-v0.md section 5.1)."""
    h = hashlib.sha256(b"g5n-conversion-v0\x00")
    for rank, manifest, records in ranks:
        p = _prepare(rank, manifest, records)
        h.update(_sha(manifest) + _sha(p["descs"]) + _sha(p["payload"]))
    return h.digest()[:16]


def build(rank, manifest, records, conv_uuid, identities=(bytes(32),) * 5) -> bytes:
    """RankFileBuilder::build + encode_rank_header (container.rs:263-315, 1037-1110)."""
    p = _prepare(rank, manifest, records)
    out = bytearray(p["pay_off"] + len(p["payload"]))
    for off, data in ((p["man_off"], manifest), (p["desc_off"], p["descs"]),
                      (p["str_off"], p["strings"]), (p["meta_off"], p["metadata"]),
                      (p["pay_off"], p["payload"])):
        out[off:off + len(data)] = data
    h = bytearray(4096)
    h[0:8] = b"GLM5NAT0"
    struct.pack_into("<HHIIIIII", h, 8, 0, 2, 4096, 0x01020304, p["flags"], rank, 4, len(records))
    struct.pack_into("<10Q", h, 40, p["man_off"], len(manifest), p["desc_off"], len(p["descs"]),
                     p["str_off"], len(p["strings"]), p["meta_off"], len(p["metadata"]),
                     p["pay_off"], len(p["payload"]))
    for i, ident in enumerate(identities):
        h[120 + 32 * i:152 + 32 * i] = ident
    h[280:312] = _sha(manifest)
    h[312:344] = _sha(p["descs"])
    h[344:376] = _sha(p["payload"])
    h[376:392] = _sha(b"g5n-file-v0\x00" + conv_uuid + struct.pack("<I", rank) + h[280:376])[:16]
    h[392:408] = conv_uuid
    h[420:452] = _sha(p["strings"])
    h[452:484] = _sha(p["metadata"])
    struct.pack_into("<I", h, 416, crc32c(bytes(h)))
    out[:4096] = h
    return bytes(out)


def resign_header(b: bytearray) -> None:
    """Recompute the header's manifest, descriptor and payload digests, file
    UUID and CRC after an edit (the reference tests' resign_header)."""
    for off_f, len_f, dst in ((40, 48, 280), (56, 64, 312), (104, 112, 344), (72, 80, 420),
                              (88, 96, 452)):
        o, n = _u64(b, off_f), _u64(b, len_f)
        b[dst:dst + 32] = _sha(b[o:o + n])
    b[376:392] = _sha(b"g5n-file-v0\x00" + bytes(b[392:408]) + bytes(b[24:28]) +
                      bytes(b[280:376]))[:16]
    b[416:420] = bytes(4)
    struct.pack_into("<I", b, 416, crc32c(bytes(b[:4096])))


# ----------------------------------------------------------------- reader
class Reader:
    """NativeRankReader::open (native_reader.rs:119-335) over in-memory bytes."""

    def __init__(self, b: bytes):
        b = bytes(b)
        self.b = b
        if len(b) < 4096:
            _fail("Truncated")
        h = b[:4096]
        flags = _u32(h, 20)
        if h[0:8] != b"GLM5NAT0" or _u16(h, 8) != 0 or _u16(h, 10) != 2 or _u32(h, 12) != 4096 or \
                _u32(h, 16) != 0x01020304 or flags & ~0x1F or _u32(h, 28) != 4 or any(h[36:40]) or \
                _u64(h, 408) != 0 or any(h[484:]):
            _fail("Header")
        chk = bytearray(h)
        chk[416:420] = bytes(4)
        if crc32c(bytes(chk)) != _u32(h, 416):
            _fail("HeaderCrc")
        self.rank = _u32(h, 24)
        if self.rank > 3:
            _fail("Rank")
        count = _u32(h, 32)
        if count == 0:
            _fail("TensorCount")

        def region(of, lf):
            s, n = _u64(h, of), _u64(h, lf)
            if s % 4096 or s + n > len(b):
                _fail("Region")
            return s, s + n
        man, desc, strs, meta, pay = (region(40, 48), region(56, 64), region(72, 80),
                                      region(88, 96), region(104, 112))
        if desc[1] - desc[0] != 256 * count or man[0] != 4096 or \
                desc[0] != _align(man[1], 4096) or strs[0] != _align(desc[1], 4096) or \
                meta[0] != _align(strs[1], 4096) or pay[0] != _align(meta[1], 4096) or \
                pay[1] != len(b):
            _fail("Region")
        for a, z in ((man[1], desc[0]), (desc[1], strs[0]), (strs[1], meta[0]), (meta[1], pay[0])):
            if any(b[a:z]):
                _fail("NonCanonicalLayout")
        if _sha(b[man[0]:man[1]]) != h[280:312] or _sha(b[desc[0]:desc[1]]) != h[312:344] or \
                _sha(b[strs[0]:strs[1]]) != h[420:452] or _sha(b[meta[0]:meta[1]]) != h[452:484]:
            _fail("StrongHash")
        self.meta_region, self.pay_region = meta, pay
        self.d, self.names, cursor = [], [], 0
        table = b[strs[0]:strs[1]]
        for i in range(count):
            d = self._decode(b[desc[0] + 256 * i:desc[0] + 256 * (i + 1)])
            if d["id"] != i or d["name_bytes"] == 0 or d["name_off"] != cursor:
                _fail("TensorId")
            raw = table[cursor:cursor + d["name_bytes"]]
            if len(raw) != d["name_bytes"]:
                _fail("StringTable")
            try:
                name = raw.decode("utf-8")
            except UnicodeDecodeError:
                _fail("StringTable")
            if any(c < 0x20 or c == 0x7F for c in raw):
                _fail("StringTable")
            self.names.append(name)
            cursor += d["name_bytes"]
            self.d.append(d)
        if cursor != len(table):
            _fail("NonCanonicalLayout")
        self._validate_descriptors()
        if header_flags([d["codec"] for d in self.d]) != flags:
            _fail("HeaderFlags")
        if _sha(b"g5n-file-v0\x00" + h[392:408] + struct.pack("<I", self.rank) + h[280:376])[:16] \
                != h[376:392]:
            _fail("FileUuid")
        self.header = h

    @staticmethod
    def _decode(b):
        """TensorDescriptor::decode (container.rs:150-213)."""
        align = _u32(b, 120)
        if any(b[25:28]) or any(b[224:]) or b[23] == 0 or b[23] > 4 or \
                bin(b[24] & 7).count("1") > 1 or align < 256 or align & (align - 1):
            _fail("Descriptor")
        ndim = b[23]
        ls = struct.unpack_from("<4I", b, 28)
        ps = struct.unpack_from("<4I", b, 44)
        if any(x == 0 for x in ls[:ndim]):
            _fail("Descriptor")
        if any(x != 1 for x in ls[ndim:]) or any(x != 1 for x in ps[ndim:]):
            _fail("Descriptor")
        if _u64(b, 64) != int(np.prod(ls[:ndim], dtype=object)):
            _fail("Descriptor")
        (tid, noff, nb, role, layer, expert, codec, ld, sd, axis, nd, flags) = \
            struct.unpack_from("<IIHHhhHHHbBB", b, 0)
        po, pb, ao, ab, mo, mb = struct.unpack_from("<6Q", b, 72)
        return dict(id=tid, name_off=noff, name_bytes=nb, role=role, layer=layer, expert=expert,
                    codec=codec, ld=ld, sd=sd, axis=axis, ndim=nd, flags=flags, ls=ls, ps=ps,
                    po=po, pb=pb, ao=ao, ab=ab, mo=mo, mb=mb, align=align, group=_u32(b, 124),
                    psha=bytes(b[128:160]), asha=bytes(b[160:192]), msha=bytes(b[192:224]))

    def _validate_descriptors(self):
        """validate_descriptors (native_reader.rs:724-858)."""
        b, meta, pay = self.b, self.meta_region, self.pay_region
        mcur, pcur = meta[0], pay[0]
        self.codec_meta = []

        def sub(s, n, parent):
            if s + n > len(b) or s < parent[0] or s + n > parent[1]:
                _fail("Region")
            return s, s + n
        for d in self.d:
            m0, m1 = sub(d["mo"], d["mb"], meta)
            if m0 != mcur:
                _fail("NonCanonicalLayout")
            mcur = m1
            cm = b[m0:m1]
            if _sha(cm) != d["msha"]:
                _fail("TensorRegion")
            p0, p1 = sub(d["po"], d["pb"], pay)
            a0, a1 = sub(d["ao"], d["ab"], pay)
            if p0 != _align(pcur, 256) or a0 != _align(p1, 256):
                _fail("NonCanonicalLayout")
            pcur = a1
            c = d["codec"]
            if c in PLAIN:
                if d["ld"] != c or d["sd"] != c or d["flags"] & 0x80 or d["group"] or d["ab"] or \
                        d["mb"]:
                    _fail("Descriptor")
                nd = d["ndim"]
                if any(d["ls"][i] == 0 or d["ls"][i] > d["ps"][i] for i in range(nd)) or \
                        int(np.prod(d["ps"][:nd], dtype=object)) * PLAIN[c] != d["pb"]:
                    _fail("Descriptor")
                self.codec_meta.append(None)
            elif c in NVFP4:
                m = nvfp4_decode(cm)
                if d["ld"] != 1 or d["sd"] != 6 or d["ndim"] != 2 or not d["flags"] & 0x80 or \
                        d["align"] != 256 or d["group"] != 16 or \
                        (m["ln"], m["lk"]) != tuple(d["ls"][:2]) or \
                        (m["pn"], m["pk"]) != tuple(d["ps"][:2]) or \
                        (0x0101 if m["two_d"] else 0x0100) != c or m["vb"] != d["pb"] or \
                        m["sb"] != d["ab"]:
                    _fail("Descriptor")
                self.codec_meta.append(m)
            elif c == EXL3:
                m = exl3_decode(cm)
                if d["layer"] < 0 or d["expert"] < 0:
                    _fail("Descriptor")
                if d["ld"] != 2 or d["sd"] != 10 or d["ndim"] != 2 or not d["flags"] & 0x80 or \
                        d["align"] != 256 or d["group"] != 0 or m["rank"] != self.rank or \
                        m["layer"] != d["layer"] or m["expert"] != d["expert"] or \
                        (m["n"], m["k"]) != tuple(d["ls"][:2]) or d["ls"] != d["ps"] or \
                        d["pb"] != 2 * m["trellis"] or d["ab"] != 2 * m["rotation"] + 4:
                    _fail("Descriptor")
                self.codec_meta.append(m)
            else:
                _fail("UnsupportedCodec")
        if mcur != meta[1] or pcur != pay[1]:
            _fail("NonCanonicalLayout")

    def planes(self, i):
        d = self.d[i]
        return self.b[d["po"]:d["po"] + d["pb"]], self.b[d["ao"]:d["ao"] + d["ab"]]

    def verify(self):
        """verify_and_stream's checks in its order (native_reader.rs:378-537)."""
        b, cursor = self.b, self.pay_region[0]
        for i, d in enumerate(self.d):
            if any(b[cursor:d["po"]]):
                _fail("NonCanonicalLayout")
            primary, aux = self.planes(i)
            c, m = d["codec"], self.codec_meta[i]
            if c in PLAIN and tuple(d["ls"]) != tuple(d["ps"]):
                nd, eb = d["ndim"], PLAIN[c]
                arr = np.frombuffer(primary, np.uint8).reshape(*d["ps"][:nd], eb)
                inside = np.ones(d["ps"][:nd], bool)
                for ax, g in enumerate(np.ix_(*[np.arange(s) for s in d["ps"][:nd]])):
                    inside &= g < d["ls"][ax]
                if np.any(arr[~inside]):
                    _fail("NonCanonicalLayout")
            if c in NVFP4:
                pn, pk, ln, lk = m["pn"], m["pk"], m["ln"], m["lk"]
                v = np.frombuffer(primary, np.uint8).reshape(pn, pk // 16, 8)
                codes = np.stack([v & 15, v >> 4], -1).reshape(pn, pk // 16, 16)
                row = np.arange(pn)[:, None]
                start = np.arange(pk // 16)[None, :] * 16
                outside = (row >= ln) | (start >= lk)
                lane_pad = (np.arange(16)[None, None, :] + start[:, :, None]) >= lk
                if np.any(codes[outside]) or np.any(codes[(~outside)[:, :, None] & lane_pad]):
                    _fail("Nvfp4(NonCanonicalPadding)")
            if _sha(primary) != d["psha"]:
                _fail("TensorRegion")
            if any(b[d["po"] + d["pb"]:d["ao"]]):
                _fail("NonCanonicalLayout")
            if c in NVFP4:
                s = np.frombuffer(aux, np.uint8)
                if np.any(s & 0x80) or np.any(s == 0x7F):
                    _fail("Nvfp4(ScaleEncoding)")
            if _sha(aux) != d["asha"]:
                _fail("TensorRegion")
            if c == EXL3:
                if _u32(aux, 0) != MCG:
                    _fail("Exl3(CodebookMarker)")
                rot = np.frombuffer(aux[4:], "<u2")
                if np.any((rot & 0x7C00) == 0x7C00):
                    _fail("Exl3(NonFiniteRotation)")
            if c in NVFP4:
                nvfp4_validate_planes(m, primary, aux)
            cursor = d["ao"] + d["ab"]
        if cursor != self.pay_region[1]:
            _fail("NonCanonicalLayout")
        if _sha(b[self.pay_region[0]:self.pay_region[1]]) != self.header[344:376]:
            _fail("StrongHash")


def validate_rank_set(readers) -> None:
    """validate_rank_set (native_reader.rs:543-588) without manifest semantics."""
    r0 = readers[0]
    h = hashlib.sha256(b"g5n-conversion-v0\x00")
    keys = ("id", "role", "layer", "expert", "codec", "ld", "sd", "axis", "ndim", "flags", "ls",
            "ps", "pb", "ab", "mb", "align", "group")
    for rank, r in enumerate(readers):
        if r.rank != rank or r.header[392:408] != r0.header[392:408] or \
                r.header[120:280] != r0.header[120:280] or r.header[20:24] != r0.header[20:24] or \
                len(r.d) != len(r0.d):
            _fail("RankSet")
        for i, d in enumerate(r.d):
            if any(d[k] != r0.d[i][k] for k in keys) or r.names[i] != r0.names[i]:
                _fail("RankSet")
            m, m0 = r.codec_meta[i], r0.codec_meta[i]
            if d["codec"] in NVFP4 and any(m[k] != m0[k] for k in
                                           ("two_d", "ln", "lk", "pn", "pk", "vb", "sb")):
                _fail("RankSet")
            if d["codec"] == EXL3 and any(m[k] != m0[k] for k in
                                          ("projection", "bits", "layer", "expert", "k", "n",
                                           "trellis", "rotation")):
                _fail("RankSet")
        h.update(r.header[280:376])
    if h.digest()[:16] != r0.header[392:408]:
        _fail("RankSet")
