/*
 * glmaxx native rank-file (.g5n) reader for NVIDIA B200: C ABI.
 *
 * Replaces the reference's Rust reader of the GLM-5.2 native rank container
 * (crates/glm-format/src/native_reader.rs, NativeRankReader; container rules in
 * crates/glm-format/src/container.rs and spec/format-v0.md sections 4-19, 26):
 *
 *   glmaxx_rank_file_open              NativeRankReader::open        (native_reader.rs:119-335)
 *   glmaxx_rank_file_info / _tensor    rank, uuids, flags, descriptors, tensor_name (:337-351)
 *   glmaxx_rank_file_codec_metadata    tensor_codec_metadata         (:353-370)
 *   glmaxx_rank_file_verify_and_stream verify_and_stream with a direct-upload sink (:378-537)
 *   glmaxx_rank_file_validate_set      validate_rank_set             (:543-588)
 *
 * Opening validates the fixed header (CRC32C), the canonical region chain, the
 * control-region SHA-256 digests, every 256-byte tensor descriptor, the codec
 * metadata records and the file UUID, reading only the control regions.
 * verify_and_stream then reads the payload region once, in order, in bounded
 * chunks: it checks the whole-payload digest, every plane digest, the zero
 * padding between planes, plain-tensor padding, the NVFP4 plane semantics
 * (codes, scale encodings, zero-scale blocks, 2-D scale sharing) and the EXL3
 * codebook marker and rotations, and copies each placed plane with
 * cudaMemcpyAsync from pinned staging straight into the caller's device
 * buffers, in the layout the kernels consume (value layout 0x1201 and the
 * 128x4 scale atoms, trellis tiles as stored: no repack).  Bytes delivered to
 * the device are tentative until the call returns 0.
 *
 * The manifest region is hash-verified but its JSON is not interpreted (the
 * reference's rank_manifest.rs schema checks are control-plane validation).
 *
 * Return codes: 0 success; GLMAXX_RANK_ERR_* (negative, below) for format,
 * integrity and argument errors; a positive cudaError_t for a failed CUDA call.
 * Without placements no CUDA call is made, so verification runs on hosts
 * without a GPU.
 */
#ifndef GLMAXX_RANK_FILE_H_
#define GLMAXX_RANK_FILE_H_

#include <stdint.h>

#if defined(__cplusplus)
extern "C" {
#endif

/* Error codes.  -1010.. mirror RankFileError (container.rs:1234-1255),
 * -1100.. Nvfp4Error (nvfp4.rs:618-633), -1200.. Exl3Error (exl3.rs:640-651),
 * -1001.. NativeRankReaderError's I/O, unsafe-file, changed-file and sink arms
 * (native_reader.rs:664-671). */
enum {
  GLMAXX_RANK_OK = 0,
  GLMAXX_RANK_ERR_NULL = -1,
  GLMAXX_RANK_ERR_ARGUMENT = -2,
  GLMAXX_RANK_ERR_IO = -1001,
  GLMAXX_RANK_ERR_UNSAFE_FILE = -1002,
  GLMAXX_RANK_ERR_CHANGED = -1003,
  GLMAXX_RANK_ERR_SINK = -1004,
  GLMAXX_RANK_ERR_TRUNCATED = -1010,
  GLMAXX_RANK_ERR_HEADER = -1011,
  GLMAXX_RANK_ERR_HEADER_FLAGS = -1012,
  GLMAXX_RANK_ERR_HEADER_CRC = -1013,
  GLMAXX_RANK_ERR_RANK = -1014,
  GLMAXX_RANK_ERR_TENSOR_COUNT = -1015,
  GLMAXX_RANK_ERR_TENSOR_ID = -1016,
  GLMAXX_RANK_ERR_DESCRIPTOR = -1017,
  GLMAXX_RANK_ERR_REGION = -1018,
  GLMAXX_RANK_ERR_TENSOR_REGION = -1019,
  GLMAXX_RANK_ERR_NON_CANONICAL_LAYOUT = -1020,
  GLMAXX_RANK_ERR_STRING_TABLE = -1021,
  GLMAXX_RANK_ERR_STRONG_HASH = -1022,
  GLMAXX_RANK_ERR_FILE_UUID = -1023,
  GLMAXX_RANK_ERR_RANK_SET = -1024,
  GLMAXX_RANK_ERR_OVERFLOW = -1025,
  GLMAXX_RANK_ERR_UNSUPPORTED_CODEC = -1026,
  GLMAXX_RANK_ERR_CODEC_MISMATCH = -1027,
  GLMAXX_RANK_ERR_NVFP4_OVERFLOW = -1101,
  GLMAXX_RANK_ERR_NVFP4_INVALID_SHAPE_OR_SCALE = -1102,
  GLMAXX_RANK_ERR_NVFP4_BYTE_ACCOUNTING = -1103,
  GLMAXX_RANK_ERR_NVFP4_METADATA_LENGTH = -1104,
  GLMAXX_RANK_ERR_NVFP4_METADATA_CRC = -1105,
  GLMAXX_RANK_ERR_NVFP4_UNSUPPORTED_METADATA = -1106,
  GLMAXX_RANK_ERR_NVFP4_SCALE_ENCODING = -1107,
  GLMAXX_RANK_ERR_NVFP4_ZERO_SCALE_VALUE = -1108,
  GLMAXX_RANK_ERR_NVFP4_NON_CANONICAL_PADDING = -1109,
  GLMAXX_RANK_ERR_NVFP4_SCALE_SHARING = -1110,
  GLMAXX_RANK_ERR_NVFP4_ALLOCATION = -1111,
  GLMAXX_RANK_ERR_EXL3_METADATA_LENGTH = -1201,
  GLMAXX_RANK_ERR_EXL3_METADATA_CRC = -1202,
  GLMAXX_RANK_ERR_EXL3_UNSUPPORTED_CONTRACT = -1203,
  GLMAXX_RANK_ERR_EXL3_CODEBOOK_MARKER = -1204,
  GLMAXX_RANK_ERR_EXL3_BYTE_ACCOUNTING = -1205,
  GLMAXX_RANK_ERR_EXL3_NON_FINITE_ROTATION = -1206,
  GLMAXX_RANK_ERR_EXL3_OVERFLOW = -1207,
};

/* Codec identifiers (format-v0.md section 9) and header flag bits (section 5). */
enum {
  GLMAXX_CODEC_BF16 = 0x0001,
  GLMAXX_CODEC_FP16 = 0x0002,
  GLMAXX_CODEC_FP32 = 0x0003,
  GLMAXX_CODEC_NVFP4_1D = 0x0100,
  GLMAXX_CODEC_NVFP4_2D = 0x0101,
  GLMAXX_CODEC_EXL3_SOURCE = 0x0200,
  GLMAXX_RANK_FLAG_DIRECT_KERNEL = 1u << 0,
  GLMAXX_RANK_FLAG_NVFP4 = 1u << 1,
  GLMAXX_RANK_FLAG_EXL3 = 1u << 2,
  GLMAXX_RANK_FLAG_HYBRID = 1u << 4,
};

/* verify_and_stream flags.  EXL3 source tensors may be placed only with
 * GLMAXX_RANK_LOAD_EXL3_SOURCE: the format keeps codec 0x0200 an inspection
 * codec (format-v0.md section 17); this library's EXL3 kernels consume the
 * source trellis layout as stored.  With GLMAXX_RANK_LOAD_HOST_DESTINATIONS
 * the dst[] addresses are host memory, filled with memcpy and no CUDA call. */
enum {
  GLMAXX_RANK_LOAD_EXL3_SOURCE = 1u << 0,
  GLMAXX_RANK_LOAD_HOST_DESTINATIONS = 1u << 1,
};

typedef struct glmaxx_rank_file glmaxx_rank_file; /* opaque */

/* Fixed-header identity of an opened file (format-v0.md section 5). */
typedef struct glmaxx_rank_file_info {
  uint32_t rank;
  uint32_t tensor_count;
  uint32_t header_flags;
  uint32_t reserved0;
  uint64_t file_bytes;
  uint64_t payload_offset;
  uint64_t payload_bytes;
  uint8_t conversion_uuid[16];
  uint8_t file_uuid[16];
  uint8_t model_config_sha256[32];
  uint8_t tokenizer_bundle_sha256[32];
  uint8_t chat_template_sha256[32];
  uint8_t weight_policy_sha256[32];
  uint8_t kernel_abi_sha256[32];
  uint8_t manifest_sha256[32];
  uint8_t descriptor_sha256[32];
  uint8_t payload_sha256[32];
} glmaxx_rank_file_info;

/* One decoded 256-byte tensor descriptor (format-v0.md section 7,
 * container.rs TensorDescriptor) plus the kernel-facing codec fields. */
typedef struct glmaxx_rank_tensor_info {
  uint32_t tensor_id;
  uint16_t role_id;
  int16_t layer_id;
  int16_t expert_id;
  uint16_t codec_id;
  uint16_t logical_dtype;
  uint16_t stored_dtype;
  int8_t tp_shard_axis;
  uint8_t ndim;
  uint8_t flags;
  uint8_t exl3_projection; /* 1 gate, 2 up, 3 down (codec 0x0200), else 0 */
  uint32_t logical_shape[4];
  uint32_t padded_shape[4];
  uint64_t payload_offset;
  uint64_t payload_bytes;
  uint64_t aux_offset;
  uint64_t aux_bytes;
  uint64_t codec_metadata_offset;
  uint64_t codec_metadata_bytes;
  uint32_t payload_alignment;
  uint32_t quant_group_elements;
  float global_scale; /* NVFP4 metadata global scale, else 0 */
  float global_amax;  /* NVFP4 metadata recorded amax, else 0 */
  const char* name;   /* string-table bytes, not NUL-terminated; valid until close */
  uint32_t name_bytes;
  uint32_t reserved1;
} glmaxx_rank_tensor_info;

/* Device destination of one tensor's planes.  The meaning of dst[] follows
 * the codec; a zero address skips that plane (it is still verified):
 *   plain (0x0001-0x0003): dst[0] = payload bytes (padded row-major)
 *   NVFP4 (0x0100/0x0101): dst[0] = value plane, dst[1] = swizzled scale plane,
 *                          dst[2] = fp32 global scale (4 bytes)
 *   EXL3  (0x0200):        dst[0] = trellis words, dst[1] = suh (K fp16),
 *                          dst[2] = svh (N fp16); the codebook marker is checked
 * dst_bytes[i] is the capacity at dst[i]; a placement whose plane is larger
 * than its capacity is refused (GLMAXX_RANK_ERR_ARGUMENT) before any copy. */
typedef struct glmaxx_rank_placement {
  uint32_t tensor_index;
  uint32_t reserved;
  uint64_t dst[3];
  uint64_t dst_bytes[3];
} glmaxx_rank_placement;

/* RankPayloadProof (native_reader.rs:653-662) plus the load's own accounting. */
typedef struct glmaxx_rank_payload_proof {
  uint32_t rank;
  uint32_t tensor_count;
  uint64_t payload_bytes;
  uint8_t payload_sha256[32];
  uint64_t stream_chunks;
  uint64_t maximum_reader_scratch_bytes;
  uint64_t storage_read_nanoseconds;
  uint64_t device_bytes; /* bytes copied to device destinations */
  uint64_t elapsed_nanoseconds;
} glmaxx_rank_payload_proof;

/* A streaming sink (RankTensorSink, native_reader.rs:606-622): called from one
 * thread in canonical tensor order -- begin_tensor, the primary plane's chunks,
 * the aux plane's chunks, finish_tensor -- with chunks of at most 8 MiB.  A
 * nonzero return stops the stream with GLMAXX_RANK_ERR_SINK.  Received bytes
 * are tentative until verify_and_stream returns 0. */
typedef struct glmaxx_rank_sink {
  void* user;
  int32_t (*begin_tensor)(void* user, uint32_t rank, uint32_t index,
                          const glmaxx_rank_tensor_info* info);
  int32_t (*primary_chunk)(void* user, const uint8_t* bytes, uint64_t length);
  int32_t (*aux_chunk)(void* user, const uint8_t* bytes, uint64_t length);
  int32_t (*finish_tensor)(void* user);
} glmaxx_rank_sink;

int32_t glmaxx_rank_file_open(const char* path, glmaxx_rank_file** out);
void glmaxx_rank_file_close(glmaxx_rank_file* file);
int32_t glmaxx_rank_file_info_get(const glmaxx_rank_file* file, glmaxx_rank_file_info* out);
int32_t glmaxx_rank_file_tensor(const glmaxx_rank_file* file, uint32_t index,
                                glmaxx_rank_tensor_info* out);
int32_t glmaxx_rank_file_codec_metadata(const glmaxx_rank_file* file, uint32_t index,
                                        const uint8_t** bytes, uint64_t* length);
/* The manifest region's bytes as read and digest-checked at open (valid until close). */
int32_t glmaxx_rank_file_manifest(const glmaxx_rank_file* file, const uint8_t** bytes,
                                  uint64_t* length);
/* Streams the payload region; placements may be NULL when count is 0.
 * stream is a cudaStream_t (NULL: the legacy default stream).  Returns after
 * every copy has completed. */
int32_t glmaxx_rank_file_verify_and_stream(const glmaxx_rank_file* file,
                                           const glmaxx_rank_placement* placements,
                                           uint32_t count, uint32_t flags, void* stream,
                                           glmaxx_rank_payload_proof* proof);
/* verify_and_stream into a caller sink instead of placements (every callback
 * may be NULL). */
int32_t glmaxx_rank_file_verify_and_stream_sink(const glmaxx_rank_file* file,
                                                const glmaxx_rank_sink* sink,
                                                glmaxx_rank_payload_proof* proof);
/* Four opened files, rank order 0..3. */
int32_t glmaxx_rank_file_validate_set(const glmaxx_rank_file* const files[4]);
const char* glmaxx_rank_file_error_name(int32_t code);

/* Nvfp4Metadata::decode plus validate_nvfp4_planes (nvfp4.rs:84-126, 466-482)
 * on in-memory planes: the check a writer runs before serialising a tensor. */
int32_t glmaxx_rank_nvfp4_validate(const uint8_t* metadata, uint64_t metadata_bytes,
                                   const uint8_t* values, uint64_t value_bytes,
                                   const uint8_t* scales, uint64_t scale_bytes);

/* The integrity primitives the reader uses (SHA-256, FIPS 180-4; CRC32C,
 * crates/glm-format/src/crc32c.rs), exported for tests and tools. */
void glmaxx_sha256(const void* data, uint64_t length, uint8_t digest[32]);
uint32_t glmaxx_crc32c(const void* data, uint64_t length);
/* 1 when the x86 SHA extensions are in use, 0 for the portable rounds;
 * glmaxx_sha256_force_portable(1) selects the portable rounds (tests). */
int32_t glmaxx_sha256_accelerated(void);
void glmaxx_sha256_force_portable(int32_t on);

#if defined(__cplusplus)
}
#endif

#endif /* GLMAXX_RANK_FILE_H_ */
