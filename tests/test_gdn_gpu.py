"""GPU: lisa_attn_gdn_recurrence (gdn_recurrence, src/kernels/shaders/
gdn.metal:245-330) against the numpy oracle, and the reference's own
invariant (tests/gdn_recurrence_state.rs:70-175): one call over 16 tokens
equals 16 one-token calls bit for bit, outputs and state, on that test's
deterministic inputs."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import lisa_attn  # noqa: E402

KH, VH, D = 16, 48, 128
KEY_DIM, VALUE_DIM = KH * D, VH * D
CONV_DIM = 2 * KEY_DIM + VALUE_DIM


def reference_inputs(steps):
    """tests/gdn_recurrence_state.rs:76-97."""
    idx = np.arange(steps * CONV_DIM)
    conv = np.where(idx % CONV_DIM < 2 * KEY_DIM, 0.0, ((idx % 127) - 63.0) * 0.002).astype(np.float32)
    qi, bi = np.arange(steps * KEY_DIM), np.arange(steps * VH)
    q = (((qi % 61) - 30.0) * 0.00002).astype(np.float32)
    k = (((qi % 67) - 33.0) * 0.0002).astype(np.float32)
    beta = (0.35 + (bi % 11) * 0.01).astype(np.float32)
    decay = (0.91 + (bi % 7) * 0.005).astype(np.float32)
    return (conv.reshape(steps, CONV_DIM), q.reshape(steps, KEY_DIM), k.reshape(steps, KEY_DIM),
            beta.reshape(steps, VH), decay.reshape(steps, VH))


def random_inputs(rng, steps):
    conv = rng.standard_normal((steps, CONV_DIM)).astype(np.float32)
    q = (rng.standard_normal((steps, KEY_DIM)) / np.sqrt(D) / D).astype(np.float32)
    k = (rng.standard_normal((steps, KEY_DIM)) / np.sqrt(D)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((steps, VH))))).astype(np.float32)
    decay = np.exp(-np.abs(rng.standard_normal((steps, VH))) * 0.1).astype(np.float32)
    return conv, q, k, beta, decay


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run(inputs, state, slots=False):
    conv, q, k, beta, decay = (cuda(a) for a in inputs)
    st = cuda(state.astype(np.float32))
    y = torch.empty((conv.shape[0], VALUE_DIM), dtype=torch.float32, device="cuda")
    sl = torch.empty((conv.shape[0], VH * D * D), dtype=torch.float32, device="cuda") if slots else None
    lisa_attn.gdn_recurrence(conv, q, k, beta, decay, st, y, VH, VH // KH, sl)
    torch.cuda.synchronize()
    return y.cpu().numpy(), st.cpu().numpy(), (sl.cpu().numpy() if slots else None)


def test_batch_equals_sequential_decode_bit_exact():
    steps = 16
    inputs = reference_inputs(steps)
    zero = np.zeros((VH, D, D), np.float32)
    yb, sb, _ = run(inputs, zero)
    state = zero
    ys = []
    for t in range(steps):
        y1, state, _ = run(tuple(a[t:t + 1] for a in inputs), state)
        ys.append(y1)
    assert np.array_equal(yb, np.concatenate(ys))
    assert np.array_equal(sb, state)
    yo, so = O.gdn_recurrence(*inputs, zero)
    assert np.abs(yb - yo).max() <= 2 ** -7 * np.abs(yo).max() + 1e-7
    assert np.abs(sb - so).max() <= 1e-5 * np.abs(so).max() + 1e-9


@pytest.mark.parametrize("steps", [1, 3, 64])
def test_random_against_oracle_with_state_slots(steps):
    rng = np.random.default_rng(500 + steps)
    inputs = random_inputs(rng, steps)
    state0 = (0.1 * rng.standard_normal((VH, D, D))).astype(np.float32)
    y, st, slots = run(inputs, state0, slots=True)
    yo, so = O.gdn_recurrence(*inputs, state0)
    # y is rounded to bf16: at most one bf16 step apart
    assert np.all(np.abs(y - yo) <= 2 ** -7 * np.abs(yo) + 1e-6)
    assert np.abs(st - so).max() <= 1e-5 * np.abs(so).max() + 1e-8
    assert np.array_equal(slots[-1].reshape(VH, D, D), st)
    if steps > 1:
        _, s1 = O.gdn_recurrence(*(a[:1] for a in inputs), state0)
        assert np.abs(slots[0].reshape(VH, D, D) - s1).max() <= 1e-5 * np.abs(s1).max() + 1e-8


def test_gdn_argument_errors():
    lib = lisa_attn.load_library()
    t = torch.zeros(16, device="cuda")
    args = [1, 48, 3] + [t.data_ptr()] * 7 + [None, 0, None]
    bad = list(args)
    bad[2] = 5  # 48 value heads not a multiple of repeat 5
    assert lib.lisa_attn_gdn_recurrence(*bad) == lisa_attn.EINVAL
    bad = list(args)
    bad[0] = 0
    assert lib.lisa_attn_gdn_recurrence(*bad) == lisa_attn.EINVAL
    bad = list(args)
    bad[11] = 16  # slot stride below one state
    bad[10] = t.data_ptr()
    assert lib.lisa_attn_gdn_recurrence(*bad) == lisa_attn.EINVAL
