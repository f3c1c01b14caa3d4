"""The decode engine's greedy pick (tc_argmax, the kernel the engine runs after the head) against
np.argmax, which the reference's lowering and board runtime call on the logits (llm.py:834,
tars_board.py:355): the first maximum, the first NaN over every number, ties, signed zeros,
denormals, infinities, whole rows of -inf, and vocabulary sizes that are not multiples of 4."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _rows(vocab, rng):
    """Rows with the cases the pick must get right, plus random rows (positions taken modulo the
    vocabulary, so tiny rows hold the cases too; the expected pick is np.argmax's either way)."""
    ix = lambda *js: [j % vocab for j in js]  # noqa: E731
    rows = [rng.normal(0, 3, vocab).astype(np.float32) for _ in range(6)]
    r = rng.normal(0, 1, vocab).astype(np.float32)
    r[ix(vocab // 3, vocab - 1, 5)] = 9.0                        # tie: the first index wins
    rows.append(r)
    r = rng.normal(0, 1, vocab).astype(np.float32)
    r[ix(7)] = 1e30
    r[ix(vocab // 2, vocab - 2)] = np.nan                      # the first NaN wins over 1e30
    rows.append(r)
    rows.append(np.full(vocab, -np.inf, np.float32))           # all -inf: index 0
    r = np.full(vocab, -np.inf, np.float32)
    r[vocab - 1] = np.inf
    rows.append(r)
    r = np.zeros(vocab, np.float32)
    r[: vocab // 2] = -0.0                                     # -0 and +0 are equal: index 0
    rows.append(r)
    r = np.full(vocab, -1.0, np.float32)
    r[ix(3, vocab - 3)] = np.frombuffer(np.uint32([1, 2]).tobytes(), np.float32)   # denormals compare exactly
    rows.append(r)
    r = rng.normal(0, 1, vocab).astype(np.float32)
    r[0] = np.nan                                              # a NaN at index 0
    rows.append(r)
    r = np.full(vocab, 2.0, np.float32)                        # a constant row: index 0
    rows.append(r)
    return np.stack(rows)


@pytest.mark.parametrize("vocab", [151936, 262144, 4096, 512, 1001, 37, 3])
def test_pick_matches_np_argmax(vocab):
    import torch

    from opentars_b200.engine import lib
    rng = np.random.default_rng(vocab)
    host = _rows(vocab, rng)
    x = torch.from_numpy(host).cuda()
    out = torch.full((host.shape[0],), -7, dtype=torch.int32, device="cuda")
    for _ in range(2):                                         # a second call on the same buffers
        rc = lib().tc_argmax(ctypes.c_void_p(x.data_ptr()), vocab, host.shape[0], ctypes.c_void_p(out.data_ptr()),
                             None)
        assert rc == 0
        torch.cuda.synchronize()
        assert out.cpu().numpy().tolist() == [int(np.argmax(r)) for r in host]


def test_pick_rejects_bad_arguments():
    from opentars_b200.engine import lib
    assert lib().tc_argmax(None, 16, 1, None, None) == -2
