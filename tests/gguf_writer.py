"""A GGUF file writer for the tests, written from the layout pkg/gguf/reader.go
parses (separately from the library's parser): little-endian header (magic,
version u32, tensor count u64, key/value count u64), key/value pairs (u64
length + key bytes, u32 value type, value; strings u64 length + bytes,
arrays u32 element type + u64 count + elements), tensor infos (name, u32
dimension count, u64 dimensions innermost first, u32 GGML type, u64 offset
into the data section), zero padding to the alignment, then the tensor data
with every tensor starting at an aligned offset."""
import struct

(U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64) = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?", U64: "<Q", I64: "<q",
        F64: "<d"}


def enc_string(s) -> bytes:
    b = s.encode() if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


def enc_value(t: int, v, elem_type: int = None) -> bytes:
    if t == STRING:
        return enc_string(v)
    if t == ARRAY:
        et, items = elem_type, v
        out = struct.pack("<IQ", et, len(items))
        for it in items:
            if et == ARRAY:
                out += enc_value(ARRAY, it[1], it[0])
            else:
                out += enc_value(et, it)
        return out
    return struct.pack(_FMT[t], v)


def gguf_bytes(metadata, tensors, version=3, alignment=32, magic=0x46554747, extra_tensor_infos=()):
    """metadata: [(key, type, value[, elem_type])]; tensors: [(name, dims, ggml_type, data)].
    Returns (file bytes, data section offset, per-tensor offsets)."""
    out = struct.pack("<IIQQ", magic, version, len(tensors) + len(extra_tensor_infos), len(metadata))
    for m in metadata:
        key, t, v = m[0], m[1], m[2]
        out += enc_string(key) + struct.pack("<I", t) + enc_value(t, v, m[3] if len(m) > 3 else None)
    offsets, off = [], 0
    for name, dims, gt, data in tensors:
        offsets.append(off)
        out += enc_string(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", gt, off)
        off += len(data)
        off += (-off) % alignment
    for name, dims, gt, off_x in extra_tensor_infos:
        out += enc_string(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", gt, off_x)
    data_off = len(out) + (-len(out)) % alignment
    out += b"\0" * (data_off - len(out))
    for (name, dims, gt, data), o in zip(tensors, offsets):
        out += b"\0" * (data_off + o - len(out))
        out += data
    return out, data_off, offsets
