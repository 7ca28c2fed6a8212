"""GPQ8 blobs for the tests, written in the layout the Qwen-7B server reads
(tools/server/qwen7b_server.c:524-563): "GPQ8", int32 count, then per tensor
int32 key length, key, int32 ndim, int32 shape[ndim], uint8 qtype (0 F32,
1 Q8), uint64 data length, data, int32 scale count, float32 scales."""
import struct

import numpy as np


def gpq8_blob(tensors):
    """tensors: [(key, array, scales or None)]; int8 arrays are Q8 tensors."""
    out = [b"GPQ8", struct.pack("<i", len(tensors))]
    for key, arr, scales in tensors:
        k = key.encode()
        out.append(struct.pack("<i", len(k)) + k)
        out.append(struct.pack("<i", arr.ndim) + b"".join(struct.pack("<i", n) for n in arr.shape))
        q8 = arr.dtype == np.int8
        data = np.ascontiguousarray(arr, np.int8 if q8 else np.float32).tobytes()
        out.append(struct.pack("<B", 1 if q8 else 0) + struct.pack("<Q", len(data)) + data)
        sc = b"" if scales is None else np.ascontiguousarray(scales, np.float32).tobytes()
        out.append(struct.pack("<i", 0 if scales is None else len(scales)) + sc)
    return b"".join(out)
