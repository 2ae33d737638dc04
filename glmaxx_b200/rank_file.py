"""GLM-5.2 native rank files (.g5n): the native reader and a writer.

``NativeRankReader`` binds the C++ reader of libglmaxx_sm100.so
(include/glmaxx_rank_file.h) and mirrors the reference's
crates/glm-format/src/native_reader.rs NativeRankReader: ``open`` validates the
header, control regions, descriptors, codec metadata and UUID; ``verify`` and
``verify_and_stream`` read the payload once, checking every digest and the
NVFP4/EXL3 plane rules; ``load`` streams the verified planes with
cudaMemcpyAsync from pinned staging straight into device tensors in the layout
the kernels consume; ``validate_rank_set`` checks four rank files against each
other.  Errors raise ``RankFileError`` whose ``kind`` names the reference's
RankFileError / Nvfp4Error / Exl3Error variant.

``RankFileBuilder`` mirrors the reference's container writer
(crates/glm-format/src/container.rs:236-470, encode_rank_header :1037-1110):
canonical region chain, 256-byte-aligned planes, descriptor and region
digests, deterministic conversion and file UUIDs.

``load_moe_layers`` places one rank's routed-MoE tensors of the requested
layers -- router weight and bias, NVFP4 or EXL3 experts, shared expert -- in
HBM as ``RankWeights`` ready for ``RoutedMoE``, in one pass over the file.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import abi

# Codec ids (format-v0.md section 9), header flags (section 5), role ids (section 18)
CODEC_BF16, CODEC_FP16, CODEC_FP32 = 0x0001, 0x0002, 0x0003
CODEC_NVFP4_1D, CODEC_NVFP4_2D, CODEC_EXL3_SOURCE = 0x0100, 0x0101, 0x0200
FLAG_DIRECT_KERNEL, FLAG_NVFP4, FLAG_EXL3, FLAG_HYBRID = 1, 2, 4, 16
LOAD_EXL3_SOURCE, LOAD_HOST_DESTINATIONS = 1, 2
ROLE_ROUTER_WEIGHT, ROLE_ROUTER_BIAS = 0x0301, 0x0302
ROLE_ROUTED_GATE_UP, ROLE_ROUTED_DOWN = 0x0501, 0x0502
ROLE_SHARED_GATE, ROLE_SHARED_UP, ROLE_SHARED_DOWN = 0x0601, 0x0602, 0x0603
EXL3_GATE, EXL3_UP, EXL3_DOWN = 1, 2, 3
EXL3_MCG_MULTIPLIER = 0xCBAC1FED
HEADER_BYTES, DESCRIPTOR_BYTES, ALIGNMENT, PAYLOAD_ALIGNMENT = 4096, 256, 4096, 256
STREAM_CHUNK_BYTES = 8 << 20
# Pinned identities that NVFP4 metadata version 0.1 records carry (nvfp4.rs:7-14)
NVFP4_LAYOUT_SOURCE_SHA256 = bytes.fromhex(
    "598e054bef21edf94b1fd6bb1447cfa9cfcf5a5907ab370128102448dbb6d530")
NVFP4_QUANT_POLICY_SHA256 = bytes.fromhex(
    "cd909579334405ecd4cd8d9a6c2dfcba7f0124c4c4ba92bc40c976d574be05a3")

_u8, _u16, _u32, _u64 = ctypes.c_uint8, ctypes.c_uint16, ctypes.c_uint32, ctypes.c_uint64
_i8, _i16, _i32, _f32 = ctypes.c_int8, ctypes.c_int16, ctypes.c_int32, ctypes.c_float


class RankFileInfo(ctypes.Structure):
    _fields_ = [("rank", _u32), ("tensor_count", _u32), ("header_flags", _u32),
                ("reserved0", _u32), ("file_bytes", _u64), ("payload_offset", _u64),
                ("payload_bytes", _u64), ("conversion_uuid", _u8 * 16), ("file_uuid", _u8 * 16)] + \
        [(n, _u8 * 32) for n in ("model_config_sha256", "tokenizer_bundle_sha256",
                                 "chat_template_sha256", "weight_policy_sha256",
                                 "kernel_abi_sha256", "manifest_sha256", "descriptor_sha256",
                                 "payload_sha256")]


class TensorInfo(ctypes.Structure):
    _fields_ = [("tensor_id", _u32), ("role_id", _u16), ("layer_id", _i16), ("expert_id", _i16),
                ("codec_id", _u16), ("logical_dtype", _u16), ("stored_dtype", _u16),
                ("tp_shard_axis", _i8), ("ndim", _u8), ("flags", _u8), ("exl3_projection", _u8),
                ("logical_shape", _u32 * 4), ("padded_shape", _u32 * 4),
                ("payload_offset", _u64), ("payload_bytes", _u64), ("aux_offset", _u64),
                ("aux_bytes", _u64), ("codec_metadata_offset", _u64),
                ("codec_metadata_bytes", _u64), ("payload_alignment", _u32),
                ("quant_group_elements", _u32), ("global_scale", _f32), ("global_amax", _f32),
                ("name", ctypes.c_void_p), ("name_bytes", _u32), ("reserved1", _u32)]


class Placement(ctypes.Structure):
    _fields_ = [("tensor_index", _u32), ("reserved", _u32), ("dst", _u64 * 3),
                ("dst_bytes", _u64 * 3)]


class PayloadProof(ctypes.Structure):
    """RankPayloadProof (native_reader.rs:653-662) plus the load's accounting."""
    _fields_ = [("rank", _u32), ("tensor_count", _u32), ("payload_bytes", _u64),
                ("payload_sha256", _u8 * 32), ("stream_chunks", _u64),
                ("maximum_reader_scratch_bytes", _u64), ("storage_read_nanoseconds", _u64),
                ("device_bytes", _u64), ("elapsed_nanoseconds", _u64)]


_BEGIN = ctypes.CFUNCTYPE(_i32, ctypes.c_void_p, _u32, _u32, ctypes.POINTER(TensorInfo))
_CHUNK = ctypes.CFUNCTYPE(_i32, ctypes.c_void_p, ctypes.POINTER(_u8), _u64)
_FINISH = ctypes.CFUNCTYPE(_i32, ctypes.c_void_p)


class _Sink(ctypes.Structure):
    _fields_ = [("user", ctypes.c_void_p), ("begin_tensor", _BEGIN), ("primary_chunk", _CHUNK),
                ("aux_chunk", _CHUNK), ("finish_tensor", _FINISH)]


_lib = None


def _load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        lib = abi.load()
        vp, pp = ctypes.c_void_p, ctypes.POINTER
        for name, res, args in [
            ("glmaxx_rank_file_open", _i32, [ctypes.c_char_p, pp(vp)]),
            ("glmaxx_rank_file_close", None, [vp]),
            ("glmaxx_rank_file_info_get", _i32, [vp, pp(RankFileInfo)]),
            ("glmaxx_rank_file_tensor", _i32, [vp, _u32, pp(TensorInfo)]),
            ("glmaxx_rank_file_codec_metadata", _i32, [vp, _u32, pp(vp), pp(_u64)]),
            ("glmaxx_rank_file_manifest", _i32, [vp, pp(vp), pp(_u64)]),
            ("glmaxx_rank_file_verify_and_stream", _i32,
             [vp, pp(Placement), _u32, _u32, vp, pp(PayloadProof)]),
            ("glmaxx_rank_file_verify_and_stream_sink", _i32, [vp, pp(_Sink), pp(PayloadProof)]),
            ("glmaxx_rank_file_validate_set", _i32, [pp(vp)]),
            ("glmaxx_rank_file_error_name", ctypes.c_char_p, [_i32]),
            ("glmaxx_rank_nvfp4_validate", _i32, [vp, _u64, vp, _u64, vp, _u64]),
            ("glmaxx_sha256", None, [vp, _u64, pp(_u8)]),
            ("glmaxx_crc32c", _u32, [vp, _u64]),
            ("glmaxx_sha256_accelerated", _i32, []),
            ("glmaxx_sha256_force_portable", None, [_i32]),
        ]:
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, args
        _lib = lib
    return _lib


class RankFileError(RuntimeError):
    """A reader or writer error; ``kind`` is the reference error variant name
    (e.g. "StrongHash", "Nvfp4(ZeroScaleValue)", "Manifest(NonCanonical)")."""

    def __init__(self, code: int, kind: str | None = None):
        self.code = code
        self.kind = kind if kind is not None else error_name(code)
        super().__init__(f"rank file error {self.kind} ({code})")


def error_name(code: int) -> str:
    return _load().glmaxx_rank_file_error_name(code).decode()


def _check(code: int) -> None:
    if code != 0:
        raise RankFileError(code)


def _buf(data) -> tuple[ctypes.c_void_p, int, object]:
    arr = np.ascontiguousarray(np.frombuffer(data, dtype=np.uint8) if isinstance(
        data, (bytes, bytearray, memoryview)) else np.asarray(data).view(np.uint8).reshape(-1))
    return ctypes.c_void_p(arr.ctypes.data), arr.nbytes, arr


def sha256(data) -> bytes:
    """SHA-256 through the library (SHA extensions when present)."""
    p, n, keep = _buf(data)
    out = (_u8 * 32)()
    _load().glmaxx_sha256(p, n, out)
    del keep
    return bytes(out)


def crc32c(data) -> int:
    p, n, keep = _buf(data)
    r = int(_load().glmaxx_crc32c(p, n))
    del keep
    return r


def sha256_accelerated() -> bool:
    return bool(_load().glmaxx_sha256_accelerated())


def sha256_force_portable(on: bool) -> None:
    _load().glmaxx_sha256_force_portable(int(on))


@dataclass
class TensorDescriptor:
    """A decoded tensor descriptor (format-v0.md section 7)."""
    tensor_id: int
    name: str
    role_id: int
    layer_id: int
    expert_id: int
    codec_id: int
    logical_dtype: int
    stored_dtype: int
    tp_shard_axis: int
    ndim: int
    flags: int
    logical_shape: tuple
    padded_shape: tuple
    payload_offset: int
    payload_bytes: int
    aux_offset: int
    aux_bytes: int
    codec_metadata_offset: int
    codec_metadata_bytes: int
    payload_alignment: int
    quant_group_elements: int
    global_scale: float
    global_amax: float
    exl3_projection: int


def _descriptor(t: TensorInfo) -> TensorDescriptor:
    return TensorDescriptor(
        t.tensor_id, ctypes.string_at(t.name, t.name_bytes).decode(), t.role_id, t.layer_id,
        t.expert_id, t.codec_id, t.logical_dtype, t.stored_dtype, t.tp_shard_axis, t.ndim,
        t.flags, tuple(t.logical_shape), tuple(t.padded_shape), t.payload_offset, t.payload_bytes,
        t.aux_offset, t.aux_bytes, t.codec_metadata_offset, t.codec_metadata_bytes,
        t.payload_alignment, t.quant_group_elements, t.global_scale, t.global_amax,
        t.exl3_projection)


def _destination(a) -> tuple[int, int]:
    """(address, capacity in bytes) of a placement destination."""
    if a is None or (isinstance(a, int) and a == 0):
        return 0, 0
    if isinstance(a, tuple):
        return int(a[0]), int(a[1])
    if isinstance(a, np.ndarray):
        if not a.flags["C_CONTIGUOUS"]:
            raise ValueError("placement destination must be contiguous")
        return a.ctypes.data, a.nbytes
    if hasattr(a, "data_ptr"):  # torch tensor
        if not a.is_contiguous():
            raise ValueError("placement destination must be contiguous")
        return a.data_ptr(), a.numel() * a.element_size()
    raise TypeError("placement destination: tensor, array, (address, bytes) or None")


def _canonical_json(raw: bytes) -> bool:
    """The manifest's bytes equal its compact, key-sorted serialisation
    (validate_rank_manifest's canonical check, rank_manifest.rs:152-157)."""
    try:
        value = json.loads(raw.decode("utf-8"))
    except (UnicodeDecodeError, ValueError):
        return False
    return json.dumps(value, separators=(",", ":"), sort_keys=True,
                      ensure_ascii=False).encode("utf-8") == raw


class NativeRankReader:
    """One opened, validated rank file (NativeRankReader::open,
    native_reader.rs:119-335)."""

    def __init__(self, path, handle: ctypes.c_void_p):
        self.path = Path(path)
        self._h = handle
        info = RankFileInfo()
        _check(_load().glmaxx_rank_file_info_get(self._h, ctypes.byref(info)))
        self.rank = info.rank
        self.header_flags = info.header_flags
        self.conversion_uuid = bytes(info.conversion_uuid)
        self.file_uuid = bytes(info.file_uuid)
        for n in ("model_config_sha256", "tokenizer_bundle_sha256", "chat_template_sha256",
                  "weight_policy_sha256", "kernel_abi_sha256", "manifest_sha256",
                  "descriptor_sha256", "payload_sha256"):
            setattr(self, n, bytes(getattr(info, n)))
        self.file_bytes, self._payload_bytes = info.file_bytes, info.payload_bytes
        self.descriptors = []
        for i in range(info.tensor_count):
            t = TensorInfo()
            _check(_load().glmaxx_rank_file_tensor(self._h, i, ctypes.byref(t)))
            self.descriptors.append(_descriptor(t))

    @classmethod
    def open(cls, path) -> "NativeRankReader":
        h = ctypes.c_void_p()
        _check(_load().glmaxx_rank_file_open(str(path).encode(), ctypes.byref(h)))
        reader = cls(path, h)
        p, n = ctypes.c_void_p(), _u64()
        _check(_load().glmaxx_rank_file_manifest(h, ctypes.byref(p), ctypes.byref(n)))
        manifest = ctypes.string_at(p, n.value) if n.value else b""
        if not _canonical_json(manifest):
            reader.close()
            raise RankFileError(0, "Manifest(NonCanonical)")
        reader.manifest = manifest
        return reader

    def close(self) -> None:
        if self._h:
            _load().glmaxx_rank_file_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tensor_count(self) -> int:
        return len(self.descriptors)

    def file_payload_bytes(self) -> int:
        return self._payload_bytes

    def tensor_name(self, index: int) -> str:
        if not 0 <= index < len(self.descriptors):
            raise RankFileError(-1016)
        return self.descriptors[index].name

    def tensor_codec_metadata(self, index: int) -> bytes:
        p, n = ctypes.c_void_p(), _u64()
        _check(_load().glmaxx_rank_file_codec_metadata(self._h, index, ctypes.byref(p),
                                                       ctypes.byref(n)))
        return ctypes.string_at(p, n.value) if n.value else b""

    def find(self, role: int, layer: int, expert: int = -1, projection: int = 0) -> list[int]:
        """Indices of the tensors with this role, layer and expert (and EXL3 projection)."""
        return [i for i, d in enumerate(self.descriptors)
                if d.role_id == role and d.layer_id == layer and d.expert_id == expert and
                (not projection or d.exl3_projection == projection)]

    def verify(self) -> PayloadProof:
        return self.load([])

    def load(self, placements, stream=None, *, exl3_source: bool = False,
             host: bool = False) -> PayloadProof:
        """verify_and_stream with a direct-upload sink: each placement is
        (tensor_index, dst0, dst1, dst2) where a destination is a torch tensor
        or numpy array (its storage and byte size), an (address, bytes) pair,
        or None to skip -- device memory, or host memory when host=True.  A
        destination smaller than its plane is refused before any copy.
        Returns after every copy completed; on an error the destinations hold
        tentative bytes."""
        arr = (Placement * max(1, len(placements)))()
        for i, (t, *dst) in enumerate(placements):
            arr[i].tensor_index = t
            for j, a in enumerate(dst):
                ptr, nbytes = _destination(a)
                arr[i].dst[j], arr[i].dst_bytes[j] = ptr, nbytes
        flags = (LOAD_EXL3_SOURCE if exl3_source else 0) | (LOAD_HOST_DESTINATIONS if host else 0)
        if stream is None and placements and not host:
            import torch
            stream = torch.cuda.current_stream().cuda_stream
        proof = PayloadProof()
        _check(_load().glmaxx_rank_file_verify_and_stream(
            self._h, arr, len(placements), flags, ctypes.c_void_p(stream or 0),
            ctypes.byref(proof)))
        return proof

    def verify_and_stream(self, sink) -> PayloadProof:
        """Stream into a Python sink with begin_tensor(rank, index, name,
        descriptor), primary_chunk(bytes), aux_chunk(bytes) and finish_tensor()
        (RankTensorSink, native_reader.rs:606-622).  A method that raises or
        returns a string stops the stream with kind "Sink"."""
        state = {"error": None}

        def guard(fn, *args):
            try:
                r = fn(*args)
                if isinstance(r, str):
                    state["error"] = r
                    return 1
                return 0
            except Exception as e:  # noqa: BLE001 -- reported as the sink's failure
                state["error"] = str(e)
                return 1

        begin = _BEGIN(lambda u, rank, idx, info: guard(
            sink.begin_tensor, rank, idx, self.descriptors[idx].name, self.descriptors[idx]))
        primary = _CHUNK(lambda u, p, n: guard(sink.primary_chunk, ctypes.string_at(p, n)))
        aux = _CHUNK(lambda u, p, n: guard(sink.aux_chunk, ctypes.string_at(p, n)))
        finish = _FINISH(lambda u: guard(sink.finish_tensor))
        s = _Sink(None, begin, primary, aux, finish)
        proof = PayloadProof()
        code = _load().glmaxx_rank_file_verify_and_stream_sink(self._h, ctypes.byref(s),
                                                               ctypes.byref(proof))
        if code != 0:
            err = RankFileError(code)
            err.message = state["error"]
            raise err
        return proof

    @staticmethod
    def validate_rank_set(readers) -> None:
        """validate_rank_set (native_reader.rs:543-588) over ranks 0..3."""
        if len(readers) != 4:
            raise RankFileError(-1024)
        arr = (ctypes.c_void_p * 4)(*[r._h for r in readers])
        _check(_load().glmaxx_rank_file_validate_set(arr))


# ====================================================================== writer
@dataclass
class PlainTensor:
    """Protected row-major tensor (format-v0.md section 10): dtype "bf16",
    "fp16" or "fp32"; data (bytes or a numpy array) covers the padded shape,
    padding zero."""
    dtype: str
    ndim: int
    logical_shape: tuple
    padded_shape: tuple
    data: bytes

    @property
    def codec(self) -> int:
        return {"bf16": CODEC_BF16, "fp16": CODEC_FP16, "fp32": CODEC_FP32}[self.dtype]


@dataclass
class Nvfp4Tensor:
    """Packed NVFP4 weight (nvfp4.rs PackedNvfp4): value plane (layout 0x1201),
    swizzled scale plane (0x1201), fp32 global scale and recorded amax."""
    logical_n: int
    logical_k: int
    padded_n: int
    padded_k: int
    global_scale: float
    global_amax: float
    values: bytes
    scales: bytes
    two_d: bool = False

    def metadata(self) -> bytes:
        """Nvfp4Metadata::encode (nvfp4.rs:40-78), 128 bytes."""
        b = bytearray(128)
        struct.pack_into("<HHHBBIIIIHHHHBBBBffII", b, 0, 0, 1,
                         CODEC_NVFP4_2D if self.two_d else CODEC_NVFP4_1D,
                         2 if self.two_d else 1, 1, self.logical_n, self.logical_k,
                         self.padded_n, self.padded_k, 16, 16 if self.two_d else 1, 0x1201,
                         0x1201, 1, 1, 1, 1, self.global_scale, self.global_amax,
                         len(_bytes_view(self.values)), len(_bytes_view(self.scales)))
        b[56:88] = NVFP4_LAYOUT_SOURCE_SHA256
        b[88:120] = NVFP4_QUANT_POLICY_SHA256
        struct.pack_into("<I", b, 120, crc32c(bytes(b)))
        return bytes(b)


@dataclass
class Exl3Tensor:
    """EXL3 source projection (exl3.rs Exl3Trellis): int16 trellis words
    [K/16, N/16, 48], fp16 suh [K] and svh [N] as uint16 bit patterns."""
    projection: int
    layer: int
    expert: int
    rank: int
    logical_k: int
    logical_n: int
    trellis: np.ndarray
    suh: np.ndarray
    svh: np.ndarray
    bits: int = 3
    mcg_marker: int = EXL3_MCG_MULTIPLIER

    @property
    def trellis_words(self) -> int:
        return (self.logical_k // 16) * (self.logical_n // 16) * 16 * self.bits

    def metadata(self) -> bytes:
        """Exl3Metadata::encode (exl3.rs:104-122), 96 bytes."""
        b = bytearray(96)
        b[0:8] = b"GLX3TR3\0"
        struct.pack_into("<HHBBBxHHIIIQQ", b, 8, 1, 1, self.projection, self.bits, self.rank,
                         self.layer, self.expert, self.logical_k, self.logical_n,
                         EXL3_MCG_MULTIPLIER, self.trellis_words,
                         self.logical_k + self.logical_n)
        struct.pack_into("<I", b, 88, crc32c(bytes(b)))
        return bytes(b)

    def validate(self) -> None:
        """Exl3Metadata::validate and Exl3Trellis::validate (exl3.rs:72-102, 317-340)."""
        k, n = self.logical_k, self.logical_n
        if not (3 <= self.layer <= 78) or self.expert >= 256 or self.rank >= 4 or self.bits != 3 \
                or k == 0 or n == 0 or k % 128 or n % 128:
            raise RankFileError(-1203)
        expected = (6144, 512) if self.projection in (EXL3_GATE, EXL3_UP) else (512, 6144)
        if self.layer <= 77 and (k, n) != expected:
            raise RankFileError(-1203)
        if self.trellis.size != self.trellis_words or self.suh.size != k or self.svh.size != n:
            raise RankFileError(-1205)
        if self.mcg_marker != EXL3_MCG_MULTIPLIER:
            raise RankFileError(-1204)
        rot = np.concatenate([np.asarray(self.suh, np.uint16), np.asarray(self.svh, np.uint16)])
        if np.any((rot & 0x7C00) == 0x7C00):
            raise RankFileError(-1206)

    def aux_plane(self) -> bytes:
        return struct.pack("<I", self.mcg_marker) + np.asarray(self.suh, "<u2").tobytes() + \
            np.asarray(self.svh, "<u2").tobytes()


@dataclass
class TensorRecord:
    tensor_id: int
    name: str
    role_id: int
    layer_id: int
    expert_id: int
    tp_shard_axis: int
    flags: int
    payload: object


def _plain_padding_ok(t: PlainTensor) -> bool:
    """Every element outside the logical shape is zero (container.rs:899-943)."""
    eb = 4 if t.dtype == "fp32" else 2
    shape = tuple(t.padded_shape[:t.ndim])
    arr = np.frombuffer(_bytes_view(t.data), dtype=np.uint8).reshape(*shape, eb)
    inside = np.ones(shape, dtype=bool)
    for axis, grid in enumerate(np.ix_(*[np.arange(s) for s in shape])):
        inside &= grid < t.logical_shape[axis]
    return not np.any(arr[~inside])


def _bytes_view(data) -> memoryview:
    """A flat byte view of bytes-like or numpy data, without a copy."""
    if isinstance(data, np.ndarray):
        return memoryview(np.ascontiguousarray(data).view(np.uint8).reshape(-1))
    return memoryview(data).cast("B")


def _encode(record: TensorRecord, rank: int):
    """EncodedTensor::from_record (container.rs:1116-1180): codec, dtypes,
    shapes, metadata, primary and aux planes of one record."""
    p = record.payload
    if isinstance(p, PlainTensor):
        eb = 4 if p.dtype == "fp32" else 2
        lshape, pshape = tuple(p.logical_shape), tuple(p.padded_shape)
        if not 1 <= p.ndim <= 4 or any(lshape[i] == 0 or lshape[i] > pshape[i]
                                       for i in range(p.ndim)) or \
                any(lshape[i] != 1 or pshape[i] != 1 for i in range(p.ndim, 4)) or \
                int(np.prod(pshape[:p.ndim])) * eb != len(_bytes_view(p.data)):
            raise RankFileError(-1017)
        if lshape != pshape and not _plain_padding_ok(p):
            raise RankFileError(-1020)
        return dict(codec=p.codec, ldtype=p.codec, sdtype=p.codec, lshape=lshape, pshape=pshape,
                    group=0, ndim=p.ndim, aux_required=False, metadata=b"",
                    primary=_bytes_view(p.data), aux=b"")
    if isinstance(p, Nvfp4Tensor):
        meta = p.metadata()
        vals = np.frombuffer(_bytes_view(p.values), np.uint8)
        scs = np.frombuffer(_bytes_view(p.scales), np.uint8)
        _check(_load().glmaxx_rank_nvfp4_validate(
            ctypes.c_char_p(meta), len(meta), ctypes.c_void_p(vals.ctypes.data), vals.nbytes,
            ctypes.c_void_p(scs.ctypes.data), scs.nbytes))
        return dict(codec=CODEC_NVFP4_2D if p.two_d else CODEC_NVFP4_1D, ldtype=1, sdtype=6,
                    lshape=(p.logical_n, p.logical_k, 1, 1),
                    pshape=(p.padded_n, p.padded_k, 1, 1), group=16, ndim=2, aux_required=True,
                    metadata=meta, primary=_bytes_view(p.values), aux=_bytes_view(p.scales))
    if isinstance(p, Exl3Tensor):
        p.validate()
        if record.layer_id < 0 or record.expert_id < 0 or p.rank != rank or \
                p.layer != record.layer_id or p.expert != record.expert_id:
            raise RankFileError(-1017)
        shape = (p.logical_n, p.logical_k, 1, 1)
        return dict(codec=CODEC_EXL3_SOURCE, ldtype=2, sdtype=10, lshape=shape, pshape=shape,
                    group=0, ndim=2, aux_required=True, metadata=p.metadata(),
                    primary=np.asarray(p.trellis, "<u2").tobytes(), aux=p.aux_plane())
    raise TypeError(f"unsupported payload {type(p).__name__}")


def _align(v: int, a: int) -> int:
    return (v + a - 1) // a * a


@dataclass
class RankFileBuilder:
    """Writer of one rank file (RankFileBuilder, container.rs:236-470)."""
    rank: int
    manifest: bytes
    model_config_sha256: bytes = bytes(32)
    tokenizer_bundle_sha256: bytes = bytes(32)
    chat_template_sha256: bytes = bytes(32)
    weight_policy_sha256: bytes = bytes(32)
    kernel_abi_sha256: bytes = bytes(32)
    tensors: list = field(default_factory=list)

    def _prepare(self):
        if not self.tensors:
            raise RankFileError(-1015)
        manifest_off = ALIGNMENT
        descriptor_off = _align(manifest_off + len(self.manifest), ALIGNMENT)
        string_off = _align(descriptor_off + len(self.tensors) * DESCRIPTOR_BYTES, ALIGNMENT)
        strings, name_offsets = bytearray(), []
        for t in self.tensors:
            name_offsets.append(len(strings))
            strings += t.name.encode()
        metadata_off = _align(string_off + len(strings), ALIGNMENT)
        metadata, meta_locals, encoded = bytearray(), [], []
        for i, t in enumerate(self.tensors):
            if t.tensor_id != i:
                raise RankFileError(-1016)
            e = _encode(t, self.rank)
            meta_locals.append(len(metadata))
            metadata += e["metadata"]
            encoded.append(e)
        payload_off = _align(metadata_off + len(metadata), ALIGNMENT)
        # payload layout: each plane at the next 256-byte boundary, zero gaps
        planes, cursor, descriptors = [], 0, bytearray()
        for i, (t, e) in enumerate(zip(self.tensors, encoded)):
            value_local = _align(cursor, PAYLOAD_ALIGNMENT)
            scale_local = _align(value_local + len(e["primary"]), PAYLOAD_ALIGNMENT)
            planes += [(value_local, e["primary"]), (scale_local, e["aux"])]
            cursor = scale_local + len(e["aux"])
            d = bytearray(DESCRIPTOR_BYTES)
            lshape = tuple(e["lshape"])
            struct.pack_into("<IIHHhhHHHbBB", d, 0, t.tensor_id, name_offsets[i], len(t.name.encode()),
                             t.role_id, t.layer_id, t.expert_id, e["codec"], e["ldtype"],
                             e["sdtype"], t.tp_shard_axis, e["ndim"],
                             t.flags | (0x80 if e["aux_required"] else 0))
            struct.pack_into("<4I4I", d, 28, *lshape, *e["pshape"])
            struct.pack_into("<QQQQQQQII", d, 64, int(np.prod(lshape[:e["ndim"]])),
                             payload_off + value_local, len(e["primary"]),
                             payload_off + scale_local, len(e["aux"]),
                             metadata_off + meta_locals[i], len(e["metadata"]), PAYLOAD_ALIGNMENT,
                             e["group"])
            d[128:160] = hashlib.sha256(e["primary"]).digest()
            d[160:192] = hashlib.sha256(e["aux"]).digest()
            d[192:224] = hashlib.sha256(e["metadata"]).digest()
            descriptors += d
        payload_len = cursor
        whole = hashlib.sha256()
        pos = 0
        for local, data in planes:
            if local > pos:
                whole.update(bytes(local - pos))
            whole.update(data)
            pos = local + len(data)
        flags = _header_flags([e["codec"] for e in encoded])
        return dict(manifest_off=manifest_off, descriptor_off=descriptor_off,
                    string_off=string_off, metadata_off=metadata_off, payload_off=payload_off,
                    descriptors=bytes(descriptors), strings=bytes(strings),
                    metadata=bytes(metadata), planes=planes, payload_len=payload_len,
                    manifest_hash=hashlib.sha256(self.manifest).digest(),
                    descriptor_hash=hashlib.sha256(bytes(descriptors)).digest(),
                    payload_hash=whole.digest(),
                    string_hash=hashlib.sha256(bytes(strings)).digest(),
                    metadata_hash=hashlib.sha256(bytes(metadata)).digest(), flags=flags)

    @staticmethod
    def derive_conversion_uuid(builders) -> bytes:
        """conversion_uuid over the four ranks' manifest, descriptor and
        payload digests (format-v0.md section 5.1)."""
        h = hashlib.sha256(b"g5n-conversion-v0\0")
        for expected, b in enumerate(builders):
            if b.rank != expected:
                raise RankFileError(-1014)
            p = b._prepare()
            h.update(p["manifest_hash"] + p["descriptor_hash"] + p["payload_hash"])
        return h.digest()[:16]

    def _header(self, p, conversion_uuid: bytes) -> bytes:
        """encode_rank_header (container.rs:1037-1110)."""
        if self.rank > 3:
            raise RankFileError(-1011)
        file_uuid = hashlib.sha256(b"g5n-file-v0\0" + conversion_uuid + struct.pack("<I", self.rank) +
                                   p["manifest_hash"] + p["descriptor_hash"] +
                                   p["payload_hash"]).digest()[:16]
        h = bytearray(HEADER_BYTES)
        h[0:8] = b"GLM5NAT0"
        struct.pack_into("<HHIIIIII", h, 8, 0, 2, HEADER_BYTES, 0x01020304, p["flags"], self.rank, 4,
                         len(self.tensors))
        struct.pack_into("<10Q", h, 40, p["manifest_off"], len(self.manifest), p["descriptor_off"],
                         len(p["descriptors"]), p["string_off"], len(p["strings"]),
                         p["metadata_off"], len(p["metadata"]), p["payload_off"], p["payload_len"])
        h[120:152] = self.model_config_sha256
        h[152:184] = self.tokenizer_bundle_sha256
        h[184:216] = self.chat_template_sha256
        h[216:248] = self.weight_policy_sha256
        h[248:280] = self.kernel_abi_sha256
        h[280:312] = p["manifest_hash"]
        h[312:344] = p["descriptor_hash"]
        h[344:376] = p["payload_hash"]
        h[376:392] = file_uuid
        h[392:408] = conversion_uuid
        h[420:452] = p["string_hash"]
        h[452:484] = p["metadata_hash"]
        struct.pack_into("<I", h, 416, crc32c(bytes(h)))
        return bytes(h)

    def write(self, path, conversion_uuid: bytes) -> int:
        """Write the file; returns its size in bytes."""
        p = self._prepare()
        header = self._header(p, conversion_uuid)
        with open(path, "wb") as f:
            f.write(header)
            for off, data in ((p["manifest_off"], self.manifest),
                              (p["descriptor_off"], p["descriptors"]),
                              (p["string_off"], p["strings"]), (p["metadata_off"], p["metadata"])):
                f.write(bytes(off - f.tell()))
                f.write(data)
            f.write(bytes(p["payload_off"] - f.tell()))
            for local, data in p["planes"]:
                f.write(bytes(p["payload_off"] + local - f.tell()))
                f.write(data)
            size = f.tell()
        return size

    def build(self, conversion_uuid: bytes) -> bytes:
        p = self._prepare()
        out = bytearray(p["payload_off"] + p["payload_len"])
        out[:HEADER_BYTES] = self._header(p, conversion_uuid)
        for off, data in ((p["manifest_off"], self.manifest),
                          (p["descriptor_off"], p["descriptors"]),
                          (p["string_off"], p["strings"]), (p["metadata_off"], p["metadata"])):
            out[off:off + len(data)] = data
        for local, data in p["planes"]:
            o = p["payload_off"] + local
            out[o:o + len(data)] = data
        return bytes(out)


def _header_flags(codecs) -> int:
    """derive_header_flags (container.rs:816-844)."""
    plain = any(c in (CODEC_BF16, CODEC_FP16, CODEC_FP32) for c in codecs)
    nv = any(c in (CODEC_NVFP4_1D, CODEC_NVFP4_2D) for c in codecs)
    ex = any(c == CODEC_EXL3_SOURCE for c in codecs)
    for c in codecs:
        if c not in (CODEC_BF16, CODEC_FP16, CODEC_FP32, CODEC_NVFP4_1D, CODEC_NVFP4_2D,
                     CODEC_EXL3_SOURCE):
            raise RankFileError(-1026)
    return ((FLAG_DIRECT_KERNEL if (plain or nv) and not ex else 0) | (FLAG_NVFP4 if nv else 0) |
            (FLAG_EXL3 if ex else 0) | (FLAG_HYBRID if nv and ex else 0))


# ============================================================ MoE layer load
def load_moe_layers(reader: NativeRankReader, cfg, layers, device=None, stream=None):
    """Place the routed-MoE tensors of ``layers`` (one rank, TP shard cfg.rank)
    in HBM with one verified pass over the file; returns ({layer: RankWeights},
    PayloadProof).  Tensors are selected by role id, layer and expert
    (format-v0.md section 18); shapes must match cfg.  A layer whose routed
    experts are EXL3 (all, or some: hybrid) gets Exl3Experts; NVFP4 planes of
    EXL3 experts are zero with global scale 1 (never routed through NVFP4).
    With device="cpu" the planes are placed in host tensors (no CUDA call)."""
    import torch

    from .moe import Exl3Experts, PackedNvfp4, RankWeights

    device = torch.device(device or "cuda")
    host = device.type == "cpu"
    if not host:  # allocations, zero fills and the load on that device, from any thread
        with torch.cuda.device(device):
            return _load_moe_layers(reader, cfg, layers, device, stream, False)
    return _load_moe_layers(reader, cfg, layers, device, stream, True)


def _load_moe_layers(reader, cfg, layers, device, stream, host):
    import torch

    from .moe import Exl3Experts, PackedNvfp4, RankWeights

    E, H, Ir, Isr = cfg.experts, cfg.hidden, cfg.local_intermediate, cfg.local_shared
    out, placements, need_exl3 = {}, [], False

    def one(role, layer, expert=-1, projection=0, required=True):
        idx = reader.find(role, layer, expert, projection)
        if len(idx) > 1 or (required and not idx):
            raise ValueError(f"layer {layer} role {role:#06x} expert {expert}: "
                             f"{len(idx)} tensors")
        return idx[0] if idx else None

    def shape(i, n, k):
        d = reader.descriptors[i]
        if tuple(d.logical_shape[:2]) != (n, k) or tuple(d.padded_shape[:2]) != (n, k):
            raise ValueError(f"{d.name}: shape {d.logical_shape[:2]} (padded "
                             f"{d.padded_shape[:2]}) != {(n, k)}")
        return d

    for layer in layers:
        rw = one(ROLE_ROUTER_WEIGHT, layer)
        rb = one(ROLE_ROUTER_BIAS, layer)
        if reader.descriptors[rw].codec_id != CODEC_BF16 or \
                reader.descriptors[rb].codec_id != CODEC_FP32:
            raise ValueError(f"layer {layer}: router weight must be bf16, bias fp32")
        shape(rw, E, H)
        if reader.descriptors[rb].logical_shape[0] != E:
            raise ValueError(f"layer {layer}: bias shape")
        router_w = torch.empty((E, H), dtype=torch.bfloat16, device=device)
        bias = torch.empty(E, dtype=torch.float32, device=device)
        placements += [(rw, router_w, None, None), (rb, bias, None, None)]

        codec = torch.zeros(E, dtype=torch.uint8)
        for e in range(E):
            gu = reader.find(ROLE_ROUTED_GATE_UP, layer, e)
            if gu and reader.descriptors[gu[0]].codec_id == CODEC_EXL3_SOURCE:
                codec[e] = 1
        any_nv, any_ex = bool((codec == 0).any()), bool((codec == 1).any())
        need_exl3 |= any_ex
        w13 = w2 = ex = None
        if any_nv:
            w13 = PackedNvfp4(torch.zeros((E, 2 * Ir, H // 2), dtype=torch.uint8, device=device),
                              torch.zeros((E, 2 * Ir * H // 16), dtype=torch.uint8, device=device),
                              torch.ones(E, dtype=torch.float32, device=device),
                              torch.zeros(E, dtype=torch.float32, device=device), 2 * Ir, H)
            w2 = PackedNvfp4(torch.zeros((E, H, Ir // 2), dtype=torch.uint8, device=device),
                             torch.zeros((E, H * Ir // 16), dtype=torch.uint8, device=device),
                             torch.ones(E, dtype=torch.float32, device=device),
                             torch.zeros(E, dtype=torch.float32, device=device), H, Ir)
        if any_ex:
            words = (H // 16) * (Ir // 16) * 48
            z = lambda *s, dt=torch.int16: torch.zeros(s, dtype=dt, device=device)  # noqa: E731
            ex = Exl3Experts(z(E, words), z(E, words), z(E, words), z(E, H, dt=torch.float16),
                             z(E, Ir, dt=torch.float16), z(E, H, dt=torch.float16),
                             z(E, Ir, dt=torch.float16), z(E, Ir, dt=torch.float16),
                             z(E, H, dt=torch.float16),
                             codec.to(device) if any_nv else None)
        amax13, amax2 = np.zeros(E, np.float32), np.zeros(E, np.float32)
        for e in range(E):
            if codec[e] == 0:
                i13 = one(ROLE_ROUTED_GATE_UP, layer, e)
                i2 = one(ROLE_ROUTED_DOWN, layer, e)
                d13, d2 = shape(i13, 2 * Ir, H), shape(i2, H, Ir)
                if CODEC_NVFP4_1D != d13.codec_id or CODEC_NVFP4_1D != d2.codec_id:
                    raise ValueError(f"layer {layer} expert {e}: routed weights must be NVFP4 1D")
                amax13[e], amax2[e] = d13.global_amax, d2.global_amax
                placements += [
                    (i13, w13.values[e], w13.scales[e], w13.global_scale[e:e + 1]),
                    (i2, w2.values[e], w2.scales[e], w2.global_scale[e:e + 1])]
            else:
                for proj, role, trellis, suh, svh, kn in (
                        (EXL3_GATE, ROLE_ROUTED_GATE_UP, ex.gate_trellis, ex.gate_suh,
                         ex.gate_svh, (Ir, H)),
                        (EXL3_UP, ROLE_ROUTED_GATE_UP, ex.up_trellis, ex.up_suh, ex.up_svh,
                         (Ir, H)),
                        (EXL3_DOWN, ROLE_ROUTED_DOWN, ex.down_trellis, ex.down_suh,
                         ex.down_svh, (H, Ir))):
                    i = one(role, layer, e, proj)
                    shape(i, *kn)
                    placements.append((i, trellis[e], suh[e], svh[e]))
        if w13 is not None:
            w13.global_amax.copy_(torch.from_numpy(amax13))
            w2.global_amax.copy_(torch.from_numpy(amax2))
        shared13 = shared2 = None
        if cfg.shared_intermediate:
            ig, iu, idn = (one(ROLE_SHARED_GATE, layer), one(ROLE_SHARED_UP, layer),
                           one(ROLE_SHARED_DOWN, layer))
            for i, n, k in ((ig, Isr, H), (iu, Isr, H), (idn, H, Isr)):
                if reader.descriptors[i].codec_id != CODEC_BF16:
                    raise ValueError(f"{reader.descriptors[i].name}: shared expert must be bf16")
                shape(i, n, k)
            shared13 = torch.empty((2 * Isr, H), dtype=torch.bfloat16, device=device)
            shared2 = torch.empty((H, Isr), dtype=torch.bfloat16, device=device)
            placements += [(ig, shared13[:Isr], None, None), (iu, shared13[Isr:], None, None),
                           (idn, shared2, None, None)]
        out[layer] = RankWeights(router_w, bias, w13, w2, shared13, shared2, ex)
    if not host:
        torch.cuda.synchronize(device)  # zero fills and amax copies precede the streamed planes
    proof = reader.load(placements, stream, exl3_source=need_exl3, host=host)
    return out, proof


def moe_layer_records(weights, cfg, layer: int, first_id: int = 0) -> list:
    """One rank's routed-MoE tensors of ``layer`` as rank-file records, named
    and flagged the way the checkpoint's TP4 rank files are (format-v0.md
    sections 7, 18, 19): router weight and fp32 correction bias replicated;
    routed gate/up [2*I_r, H] column-parallel (NVFP4) or EXL3 gate, up (K=H,
    N=I_r) and down (K=I_r, N=H) projections; shared gate/up column-parallel
    and down row-parallel, bf16.  Device tensors are copied to the host."""
    E, H, Ir, Isr = cfg.experts, cfg.hidden, cfg.local_intermediate, cfg.local_shared
    out = []
    pre = f"model.layers.{layer}.mlp"

    def add(name, role, expert, axis, flags, payload):
        out.append(TensorRecord(first_id + len(out), name, role, layer, expert, axis, flags,
                                payload))

    def host(t):
        return t.detach().contiguous().cpu().numpy()

    add(f"{pre}.gate.weight", ROLE_ROUTER_WEIGHT, -1, -1, 1,
        PlainTensor("bf16", 2, (E, H, 1, 1), (E, H, 1, 1),
                    host(weights.router_weight.view(_torch_uint8()))))
    add(f"{pre}.gate.e_score_correction_bias", ROLE_ROUTER_BIAS, -1, -1, 1,
        PlainTensor("fp32", 1, (E, 1, 1, 1), (E, 1, 1, 1), host(weights.router_bias)))
    ex = weights.exl3
    codec = None if ex is None or ex.codec is None else host(ex.codec)
    for e in range(E):
        if ex is None or (codec is not None and codec[e] == 0):
            for role, p, n, k, name, axis, flags in (
                    (ROLE_ROUTED_GATE_UP, weights.w13, 2 * Ir, H, "gate_up_proj", 0, 0b1010),
                    (ROLE_ROUTED_DOWN, weights.w2, H, Ir, "down_proj", 1, 0b1100)):
                add(f"{pre}.experts.{e}.{name}.weight", role, e, axis, flags,
                    Nvfp4Tensor(n, k, n, k, float(p.global_scale[e]), float(p.global_amax[e]),
                                host(p.values[e]), host(p.scales[e])))
        else:
            for proj, role, tr, suh, svh, k, n, name, axis, flags in (
                    (EXL3_GATE, ROLE_ROUTED_GATE_UP, ex.gate_trellis, ex.gate_suh, ex.gate_svh,
                     H, Ir, "gate_proj", 0, 0b1010),
                    (EXL3_UP, ROLE_ROUTED_GATE_UP, ex.up_trellis, ex.up_suh, ex.up_svh, H, Ir,
                     "up_proj", 0, 0b1010),
                    (EXL3_DOWN, ROLE_ROUTED_DOWN, ex.down_trellis, ex.down_suh, ex.down_svh, Ir,
                     H, "down_proj", 1, 0b1100)):
                add(f"{pre}.experts.{e}.{name}.weight", role, e, axis, flags,
                    Exl3Tensor(proj, layer, e, cfg.rank, k, n, host(tr[e]).view(np.uint16),
                               host(suh[e]).view(np.uint16), host(svh[e]).view(np.uint16)))
    if weights.shared13 is not None:
        s13 = host(weights.shared13.view(_torch_uint8())).reshape(2 * Isr, H * 2)
        for role, rows, name in ((ROLE_SHARED_GATE, s13[:Isr], "gate_proj"),
                                 (ROLE_SHARED_UP, s13[Isr:], "up_proj")):
            add(f"{pre}.shared_experts.{name}.weight", role, -1, 0, 0b10010,
                PlainTensor("bf16", 2, (Isr, H, 1, 1), (Isr, H, 1, 1), rows))
        add(f"{pre}.shared_experts.down_proj.weight", ROLE_SHARED_DOWN, -1, 1, 0b10100,
            PlainTensor("bf16", 2, (H, Isr, 1, 1), (H, Isr, 1, 1),
                        host(weights.shared2.view(_torch_uint8()))))
    return out


def _torch_uint8():
    import torch
    return torch.uint8


def _set_identity(reader: NativeRankReader) -> dict:
    """What validate_rank_set compares of one file (native_reader.rs:543-588):
    rank, conversion UUID, the five input identities, header flags, the three
    region digests, and per tensor the descriptor semantics, name and codec
    semantics (NVFP4 geometry and plane sizes; EXL3 projection, shape, words)."""
    tensors = []
    for i, d in enumerate(reader.descriptors):
        codec = ()
        m = reader.tensor_codec_metadata(i)
        if d.codec_id in (CODEC_NVFP4_1D, CODEC_NVFP4_2D):
            codec = (m[6],) + struct.unpack_from("<IIII", m, 8) + struct.unpack_from("<II", m, 44)
        elif d.codec_id == CODEC_EXL3_SOURCE:
            codec = (m[12], m[13]) + struct.unpack_from("<HHII", m, 16) + \
                struct.unpack_from("<QQ", m, 32)
        tensors.append((d.tensor_id, d.role_id, d.layer_id, d.expert_id, d.codec_id,
                        d.logical_dtype, d.stored_dtype, d.tp_shard_axis, d.ndim, d.flags,
                        d.logical_shape, d.padded_shape, d.payload_bytes, d.aux_bytes,
                        d.codec_metadata_bytes, d.payload_alignment, d.quant_group_elements,
                        d.name, codec))
    return {"rank": reader.rank, "conversion_uuid": reader.conversion_uuid,
            "identities": b"".join(getattr(reader, n) for n in (
                "model_config_sha256", "tokenizer_bundle_sha256", "chat_template_sha256",
                "weight_policy_sha256", "kernel_abi_sha256")),
            "header_flags": reader.header_flags,
            "digests": reader.manifest_sha256 + reader.descriptor_sha256 + reader.payload_sha256,
            "tensors": tensors}


def validate_rank_set_distributed(reader: NativeRankReader, group=None) -> None:
    """validate_rank_set when every rank process holds only its own file: the
    four files' set identities are all-gathered over ``group`` (torch.distributed,
    world size 4) and every rank applies the same checks to the same data, so
    all ranks pass or all raise RankFileError("RankSet") together."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    gathered = [None] * world
    dist.all_gather_object(gathered, _set_identity(reader), group=group)
    if world != 4 or any(g["rank"] != r for r, g in enumerate(gathered)):
        raise RankFileError(-1024)
    first = gathered[0]
    h = hashlib.sha256(b"g5n-conversion-v0\0")
    for g in gathered:
        for key in ("conversion_uuid", "identities", "header_flags", "tensors"):
            if g[key] != first[key]:
                raise RankFileError(-1024)
        h.update(g["digests"])
    if h.digest()[:16] != first["conversion_uuid"]:
        raise RankFileError(-1024)


def load_rank_set(paths, cfgs, layers, devices):
    """A node's four TP rank files: open them, validate_rank_set, then load each
    rank's layers on its own device concurrently (one thread per file; the
    native reader runs without the GIL).  Returns ([{layer: RankWeights}] in
    rank order, [PayloadProof]).  cfgs[r] and devices[r] belong to rank r."""
    from concurrent.futures import ThreadPoolExecutor
    readers = [NativeRankReader.open(p) for p in paths]
    try:
        NativeRankReader.validate_rank_set(readers)
        with ThreadPoolExecutor(len(readers)) as pool:
            results = list(pool.map(lambda r: load_moe_layers(readers[r], cfgs[r], layers,
                                                              devices[r]), range(len(readers))))
    finally:
        for rd in readers:
            rd.close()
    return [w for w, _ in results], [p for _, p in results]
