"""Scripted stand-in for ContinuousModel in CPU tests of the service and the dispatcher.

Every request emits one 1920-sample PCM16 chunk per tick whose samples encode
(identifier, frame) and finishes after ``max_new_tokens - 1`` frames with
"length". Inputs steer failures: "crash" raises inside tick, "exit" ends the
process, "hang" stops the engine from making progress; ``start_marker`` makes
every start after the first fail.
"""
import os
import time

import numpy as np


def chunk(identifier: int, frame: int) -> bytes:
    return np.full(1920, (identifier * 100 + frame) % 30000, dtype="<i2").tobytes()


class FakeEngine:
    def __init__(self, device="cpu", start_marker=None, **kwargs):
        # start_marker: a file path; every start after the first one that created it fails
        if start_marker is not None:
            if os.path.exists(start_marker):
                raise RuntimeError("scripted start failure")
            open(start_marker, "w").close()
        self.device = device
        self.speakers, self.languages = ["ryan", "voice_a"], ["auto", "english"]
        self.active = {}
        self.closed = False

    def tick(self, submissions, emit, cancelled):
        for identifier in cancelled:
            self.active.pop(identifier, None)
        for identifier, payload in submissions:
            if payload["input"] == "crash":
                raise RuntimeError("scripted engine failure")
            if payload["input"] == "exit":
                os._exit(3)
            if payload["input"] == "hang":
                time.sleep(3600)
            self.active[identifier] = [payload, 0]
        outputs = []
        for identifier, state in list(self.active.items()):
            payload, frames = state
            pcm = chunk(identifier, frames)
            state[1] = frames + 1
            if emit is not None:
                emit(identifier, pcm, 24000)
            if state[1] >= payload["max_new_tokens"] - 1:
                data = b"".join(chunk(identifier, f) for f in range(state[1]))
                outputs.append((identifier, {"pcm": data, "sample_rate": 24000, "codec_frames": state[1],
                                             "finish_reason": "length", "device": self.device}))
                del self.active[identifier]
        time.sleep(0.002)
        return outputs

    def close(self):
        self.closed = True
