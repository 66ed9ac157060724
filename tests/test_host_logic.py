"""Host-side logic of the training loop that needs no GPU."""
import numpy as np

from gs3d.training import Trainer


def _order_only_trainer(ncams, seed):
    t = Trainer.__new__(Trainer)  # only the camera-order state
    t.cameras = list(range(ncams))
    t.rng = np.random.default_rng(seed)
    t.cameras_order = t.rng.permutation(ncams)
    t.cameras_order_idx = -1
    t._next_orders = []
    return t


def _lazy_sequence(ncams, seed, steps):
    """The camera sequence of training.jl:174-178: shuffled order, re-shuffled after each pass."""
    rng = np.random.default_rng(seed)
    order, k, out = rng.permutation(ncams), -1, []
    for _ in range(steps):
        k += 1
        if k >= ncams:
            order, k = rng.permutation(ncams), 0
        out.append(int(order[k]))
    return out


def test_peeked_cameras_follow_the_training_order():
    """Looking ahead for the target prefetch draws the coming permutations in order, so the
    cameras visited are the ones the lazy re-shuffle would give."""
    for ncams, ahead in ((1, 1), (3, 1), (7, 1), (5, 3), (4, 9)):
        t = _order_only_trainer(ncams, seed=ncams)
        want = _lazy_sequence(ncams, ncams, 40)
        got = []
        for step in range(40):
            if step + ahead < 40 and step > 0:
                peek = t.peek_camera_index(ahead)
                assert peek == want[step - 1 + ahead], (ncams, ahead, step)
            t.advance_camera()
            got.append(int(t.cameras_order[t.cameras_order_idx]))
        assert got == want, (ncams, ahead)
