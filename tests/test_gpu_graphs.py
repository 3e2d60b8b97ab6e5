"""CapturedStep: a training step recorded as a CUDA graph and replayed gives
the same parameters, bit for bit, as the same steps run eagerly."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def J():
    import jax4j_b200 as j
    return j


def _mlp_step(J, dims, act):
    neg = J.ConcreteNDArray.scalar(-1.0)
    lr = J.ConcreteNDArray.scalar(0.05)
    names = [f"{k}{i}" for i in range(1, len(dims)) for k in ("w", "b")]

    def loss(tr, x, t):
        c = tr.children
        a = x
        for i in range(1, len(dims)):
            a = a.dot(c[f"w{i}"].value).add(c[f"b{i}"].value)
            if i < len(dims) - 1:
                a = a.tanh() if act == "tanh" else a.relu()
        return J.Nn.softmax(a).log().mul(t).sum(-1).mean().mul(neg)

    def step(x, t, *ps):
        p = dict(zip(names, ps))
        new = {}

        def body(xs, ts):
            v, g = J.JAX.valueAndGradTree(lambda tr: loss(tr, xs, ts))(J.PyTree.dictOf(p))
            g = J.Lax.psumTree(g).children
            for k in names:
                new[k] = p[k].sub(g[k].value.mul(lr))
            return v

        D = x.shape().dimensions()[0]
        losses = J.JAX.pmap(body, [J.Device.defaultDevice()] + [J.Device(None) for _ in range(D - 1)])(x, t)
        return [losses] + [new[k] for k in names]

    return names, step


@pytest.mark.parametrize("dims,act,D", [([64, 48, 10], "tanh", 1), ([96, 128, 128, 20], "relu", 2)])
def test_captured_step_matches_eager(J, dims, act, D):
    from jax4j_b200.graphs import CapturedStep
    B = 32
    names, step = _mlp_step(J, dims, act)
    keys = J.Random.split(J.PRNGKey.key(7), len(dims))
    params = []
    for i in range(1, len(dims)):
        params.append(J.Random.glorotUniform(keys[i - 1], J.Shape(dims[i - 1], dims[i]), dims[i - 1], dims[i]))
        params.append(J.Random.uniform(keys[i], J.Shape(dims[i]), -0.1, 0.1))
    x = J.Random.normal(J.PRNGKey.key(1), J.Shape(D, B, dims[0]))
    lab = np.arange(D * B) * 7 % dims[-1]
    t = np.zeros((D * B, dims[-1]), np.float32)
    t[np.arange(D * B), lab] = 1
    tt = J.ConcreteNDArray.of(t.reshape(D, B, dims[-1]))

    # eager reference: three steps
    ps = [J.ConcreteNDArray._wrap(p.tensor().clone(), p.shape(), p.dtype(), p.device()) for p in params]
    eager_losses = []
    for _ in range(3):
        outs = step(x, tt, *ps)
        eager_losses.append(outs[0].numpy().copy())
        ps = outs[1:]

    # recorded once (after its warm-up, which does not advance the parameters), replayed three times
    static = [J.ConcreteNDArray._wrap(p.tensor().clone(), p.shape(), p.dtype(), p.device()) for p in params]
    cs = CapturedStep(step, [x, tt] + static, donate={1 + j: 2 + j for j in range(len(names))})
    for i in range(3):
        out = cs()
        np.testing.assert_array_equal(out[0].numpy(), eager_losses[i])
    for a, b in zip(cs.inputs[2:], ps):
        np.testing.assert_array_equal(a.numpy(), b.numpy())
    cs.release()


def test_captured_step_rejects_bad_donation(J):
    from jax4j_b200.graphs import CapturedStep
    a = J.ConcreteNDArray.of(np.ones(8, np.float32))
    with pytest.raises(ValueError):
        CapturedStep(lambda v: [v.add(v)], [a], donate={0: 3})
