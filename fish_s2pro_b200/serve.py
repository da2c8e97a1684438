"""Continuous batching over the batched frame: the serving layer above the
C ABI's s2d_serve_* calls.

The reference serves `/v1/tts` one request at a time: `tts_handler`
(crates/fish_s2_infer/src/server.rs:89-120) locks the engine and runs
`InferenceEngine::synthesize_wav` (engine.rs:255-287), whose pipeline calls
`generate_codes` (pipeline.rs:174-182) for the whole utterance.  Here many
requests share one batched frame: `TtsScheduler` keeps a FIFO queue, admits
requests into free slots between frames when the KV pool has their pages,
advances every running slot a few frames at a time and hands back each
finished request's codes (the codec's input; text tokenisation and the codec
stay on the host, as in the reference).
"""
from __future__ import annotations

import collections
import ctypes
import dataclasses
import time
from typing import Deque, Dict, List

import numpy as np

from .s2d import (RNG_SEEDED, DecodeProfile, GenerateCodesResult, GenerateParams, PromptTensor,
                  S2dError, SeededRng, SlowArState, _GenParams, _ptr, lib)

S2D_EFULL = -7
SLOT_FREE, SLOT_RUNNING, SLOT_FINISHED = 0, 1, 2


class ServeSession:
    """One s2d_serve_* session on a handle opened with max_batch slots.
    Every request shares `params` (and the tokenizer's im_end id)."""

    def __init__(self, state: SlowArState, im_end_id: int, params: GenerateParams,
                 rng_kind: int = RNG_SEEDED, philox_key: int = 0):
        self.state = state
        self.params = params
        self.slots = state.max_batch
        self.k = max(state.graph_spec().num_codebooks, 1)
        gp = _GenParams(params.max_new_tokens, params.temperature, params.top_p, params.top_k,
                        params.min_tokens_before_end, int(im_end_id))
        state._check(lib().s2d_serve_begin(state.handle, ctypes.byref(gp), rng_kind,
                                           ctypes.c_uint64(philox_key)))

    def admit(self, slot: int, prompt: PromptTensor, rng_state: int) -> bool:
        """Prefill `prompt` into `slot`; False when the pool lacks its pages."""
        data = np.ascontiguousarray(np.asarray(prompt.data, dtype=np.uint32).reshape(-1))
        if data.size != prompt.rows * prompt.cols:
            raise S2dError(-1, "prompt data length mismatch")
        rc = lib().s2d_serve_admit(self.state.handle, slot, _ptr(data, ctypes.c_uint32), prompt.rows,
                                   prompt.cols, ctypes.c_uint64(rng_state))
        if rc == S2D_EFULL:
            return False
        self.state._check(rc)
        return True

    def step(self, n_frames: int):
        """Advance every running slot by n_frames; returns (status, frames) per slot."""
        status = np.zeros(self.slots, dtype=np.int32)
        frames = np.zeros(self.slots, dtype=np.uint32)
        self.state._check(lib().s2d_serve_step(self.state.handle, n_frames, _ptr(status, ctypes.c_int32),
                                               _ptr(frames, ctypes.c_uint32)))
        return status, frames

    def collect(self, slot: int):
        """A finished slot's (codebook-major codes, n_frames, rng state); frees the slot."""
        codes = np.zeros(self.k * max(self.params.max_new_tokens, 1), dtype=np.int32)
        n = ctypes.c_uint32()
        rng = ctypes.c_uint64()
        self.state._check(lib().s2d_serve_collect(self.state.handle, slot, _ptr(codes, ctypes.c_int32),
                                                  ctypes.byref(n), ctypes.byref(rng)))
        return codes[: self.k * n.value].copy(), n.value, rng.value

    def free_pages(self) -> int:
        out = ctypes.c_int32()
        self.state._check(lib().s2d_serve_free_pages(self.state.handle, ctypes.byref(out)))
        return out.value


@dataclasses.dataclass
class TtsRequest:
    id: int
    prompt: PromptTensor
    rng: SeededRng
    submitted: float = 0.0
    admitted: float = 0.0
    admitted_frame: int = -1


@dataclasses.dataclass
class TtsResult:
    id: int
    result: GenerateCodesResult
    rng_state: int
    queue_s: float     # submit -> admission
    latency_s: float   # submit -> codes collected
    admitted_frame: int  # session frame at which the request joined


class TtsScheduler:
    """FIFO continuous batching: between frames, finished requests leave and
    queued ones take the free slots (in submission order; a request that
    does not fit the free KV pages waits, and so do the ones behind it)."""

    def __init__(self, state: SlowArState, im_end_id: int, params: GenerateParams,
                 rng_kind: int = RNG_SEEDED, philox_key: int = 0, frames_per_step: int = 4):
        self.session = ServeSession(state, im_end_id, params, rng_kind, philox_key)
        self.frames_per_step = max(1, int(frames_per_step))
        self.queue: Deque[TtsRequest] = collections.deque()
        self.running: Dict[int, TtsRequest] = {}
        self.frame = 0  # frames the session has run
        self._next_id = 0

    def submit(self, prompt: PromptTensor, rng: SeededRng) -> int:
        rid = self._next_id
        self._next_id += 1
        self.queue.append(TtsRequest(rid, prompt, rng, submitted=time.perf_counter()))
        return rid

    def _admit(self) -> None:
        for slot in range(self.session.slots):
            if not self.queue:
                return
            if slot in self.running:
                continue
            req = self.queue[0]
            if not self.session.admit(slot, req.prompt, req.rng.state):
                return  # the pool is short of pages: wait for a request to finish
            self.queue.popleft()
            req.admitted, req.admitted_frame = time.perf_counter(), self.frame
            self.running[slot] = req

    def step(self) -> List[TtsResult]:
        """Admit what fits, run frames_per_step frames, collect the finished."""
        self._admit()
        if not self.running:
            return []
        status, _ = self.session.step(self.frames_per_step)
        self.frame += self.frames_per_step
        done = []
        for slot in [s for s, st in enumerate(status) if st == SLOT_FINISHED]:
            req = self.running.pop(slot)
            codes, n, rng_state = self.session.collect(slot)
            req.rng.state = rng_state
            now = time.perf_counter()
            res = GenerateCodesResult(codes=codes, num_codebooks=self.session.k, n_frames=n,
                                      profile=DecodeProfile(0.0, 0.0, n, 0, 0, 0))
            done.append(TtsResult(req.id, res, rng_state, req.admitted - req.submitted, now - req.submitted,
                                  req.admitted_frame))
        return done

    def run(self) -> Dict[int, TtsResult]:
        """Serve until the queue is empty and every slot is free."""
        out: Dict[int, TtsResult] = {}
        while self.queue or self.running:
            done = self.step()
            for r in done:
                out[r.id] = r
            if not done and not self.running:  # nothing admitted into an idle session
                raise S2dError(S2D_EFULL, "a queued request needs more KV pages than the whole pool")
        return out
