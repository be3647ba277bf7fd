"""Digest of integer arrays, shared by the golden-fixture generator and the tests.

Every array is cast to little-endian int64 before hashing, so a torch int32
expert_map and a numpy int64 one with the same values give the same digest.
"""

import hashlib

import numpy as np


def digest(*arrays) -> bytes:
    h = hashlib.sha1()
    for a in arrays:
        if hasattr(a, "detach"):
            a = a.detach().cpu().numpy()
        h.update(np.ascontiguousarray(np.asarray(a), dtype="<i8").tobytes())
        h.update(b"|")
    return h.hexdigest()[:24].encode()
