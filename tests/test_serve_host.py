"""Host logic of the continuous-batching scheduler (fish_s2pro_b200.serve)
against a fake session, so that no GPU is needed: FIFO admission into free
slots, waiting while the KV pool is short of pages, collection of finished
slots, and the error for a request larger than the whole pool."""
import numpy as np
import pytest

from fish_s2pro_b200 import serve
from fish_s2pro_b200.s2d import GenerateParams, PromptTensor, S2dError, SeededRng

PAGE = 64


class FakeSession:
    """Slots that finish max_new frames after admission; pages as the C side
    counts them: ceil((cols + max_new) / 64) per request."""

    def __init__(self, state, im_end_id, params, rng_kind=0, philox_key=0):
        self.params = params
        self.slots = state.slots
        self.k = 2
        self.pages = state.pages
        self.cols = [-1] * self.slots
        self.frames = [0] * self.slots
        self.held = [0] * self.slots
        self.log = state.log

    def admit(self, slot, prompt, rng_state):
        assert self.cols[slot] < 0
        need = -(-(prompt.cols + self.params.max_new_tokens) // PAGE)
        if need > self.pages:
            return False
        self.pages -= need
        self.cols[slot], self.frames[slot], self.held[slot] = prompt.cols, 0, need
        self.log.append(("admit", slot, int(rng_state)))
        return True

    def step(self, n):
        status = np.zeros(self.slots, np.int32)
        for s in range(self.slots):
            if self.cols[s] >= 0:
                self.frames[s] = min(self.params.max_new_tokens, self.frames[s] + n)
                status[s] = 2 if self.frames[s] == self.params.max_new_tokens else 1
        return status, np.array(self.frames, np.uint32)

    def collect(self, slot):
        n = self.frames[slot]
        codes = np.full(self.k * n, slot, np.int32)
        self.pages += self.held[slot]
        self.cols[slot] = -1
        self.log.append(("collect", slot))
        return codes, n, 1000 + slot


class FakeState:
    def __init__(self, slots, pages):
        self.slots, self.pages, self.log = slots, pages, []


def prompt(cols):
    return PromptTensor(3, cols, np.zeros(3 * cols, np.uint32))


@pytest.fixture
def fake(monkeypatch):
    monkeypatch.setattr(serve, "ServeSession", FakeSession)


def test_fifo_admission_and_collection(fake):
    st = FakeState(slots=2, pages=100)
    sch = serve.TtsScheduler(st, 7, GenerateParams(8, 0.0, 1.0, 0, 20), frames_per_step=3)
    ids = [sch.submit(prompt(10 + i), SeededRng(i)) for i in range(5)]
    out = sch.run()
    assert sorted(out) == ids
    admits = [e for e in st.log if e[0] == "admit"]
    assert [e[2] for e in admits] == [0, 1, 2, 3, 4]  # submission order
    # two slots: requests 2.. join after the first ones finish (3 steps of 3 frames)
    assert [out[i].admitted_frame for i in ids] == [0, 0, 9, 9, 18]
    assert all(out[i].result.n_frames == 8 for i in ids)


def test_waits_for_pages(fake):
    # 5 pages: each request needs ceil((100 + 8) / 64) = 2, so at most 2 run at once
    st = FakeState(slots=4, pages=5)
    sch = serve.TtsScheduler(st, 7, GenerateParams(8, 0.0, 1.0, 0, 20), frames_per_step=8)
    ids = [sch.submit(prompt(100), SeededRng(i)) for i in range(5)]
    out = sch.run()
    assert [out[i].admitted_frame for i in ids] == [0, 0, 8, 8, 16]


def test_request_larger_than_pool(fake):
    st = FakeState(slots=2, pages=1)
    sch = serve.TtsScheduler(st, 7, GenerateParams(8, 0.0, 1.0, 0, 20))
    sch.submit(prompt(100), SeededRng(0))
    with pytest.raises(S2dError):
        sch.run()
