"""Binary hop frames (rtc.js:7-22): 4 x Int32 header [msgType, seqId, posStart,
nFloats] followed by an fp32 payload, little-endian as JS typed arrays are."""
from __future__ import annotations

import numpy as np


def pack(msg_type: int, seq_id: int, pos_start: int, f32) -> bytes:
    a = np.ascontiguousarray(f32, dtype="<f4").reshape(-1)
    head = np.array([msg_type, seq_id, pos_start, a.size], dtype="<i4")
    return head.tobytes() + a.tobytes()


def unpack(data: bytes) -> dict:
    n = len(data) - 16
    if n < 0 or n % 4 != 0:
        raise ValueError(f"bad frame size {len(data)}")  # rtc.js:17
    head = np.frombuffer(data, dtype="<i4", count=4)
    f32 = np.frombuffer(data, dtype="<f4", offset=16, count=n // 4).copy()
    return {"msgType": int(head[0]), "seqId": int(head[1]), "posStart": int(head[2]), "f32": f32}
