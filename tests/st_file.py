"""Writes safetensors files for the reader's tests (test helper): the
format's u64 little-endian header length, the JSON header, then the data."""
import json
import struct

import numpy as np

DT = {np.float32: "F32", np.float16: "F16", np.uint32: "U32", np.int32: "I32",
      np.uint8: "U8", np.int8: "I8", np.float64: "F64", np.int64: "I64", np.uint16: "U16",
      np.int16: "I16"}


def write(path, tensors, metadata=None, bf16=(), header_extra=None, raw_header=None):
    """tensors: name -> numpy array; names in `bf16` are uint16 bit arrays
    stored as BF16.  header_extra: entries merged into the header as is."""
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        a = np.asarray(a)
        dt = "BF16" if name in bf16 else DT[a.dtype.type]
        b = a.tobytes(order="C")
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = metadata
    if header_extra:
        header.update(header_extra)
    h = raw_header if raw_header is not None else json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
    return path
