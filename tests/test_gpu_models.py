"""The workloads of the path, end to end through the public API, against the
oracle: the MLP cross-entropy grad steps (tanh 2-layer and relu 4-layer, at
reduced sizes the oracle finishes in seconds), grad-of-pmap w.r.t. the input,
and the elementwise where/tanh/sigmoid/clip sweep with sum and argmax."""
import numpy as np
import pytest

from oracle import oracle as orc
from tests.util import TOL_ELEMENTWISE, TOL_REDUCTION, assert_rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def J():
    import jax4j_b200 as j
    return j


def make_mlp(J, dims, seed):
    """Glorot weights and zero biases from split keys (seeded like the configs)."""
    keys = J.Random.split(J.PRNGKey.key(seed), len(dims) - 1)
    tree = {}
    for i in range(len(dims) - 1):
        tree[f"w{i + 1}"] = J.Random.glorotUniform(keys[i], J.Shape(dims[i], dims[i + 1]), dims[i], dims[i + 1])
        tree[f"b{i + 1}"] = J.ConcreteNDArray.full(J.Shape(dims[i + 1]), 0.0)
    return J.PyTree.dictOf(tree)


def mlp_loss(J, act):
    def loss(p, x, t):
        c = p.children
        L = len(c) // 2
        a = x
        for i in range(1, L):
            z = a.dot(c[f"w{i}"].value).add(c[f"b{i}"].value)
            a = z.tanh() if act == "tanh" else z.relu()
        logits = a.dot(c[f"w{L}"].value).add(c[f"b{L}"].value)
        neg = J.ConcreteNDArray.scalar(-1.0, device=x.device())
        return J.Nn.softmax(logits).log().mul(t).sum(-1).mean().mul(neg)
    return loss


def onehot(labels, C):
    t = np.zeros((len(labels), C), np.float32)
    t[np.arange(len(labels)), labels] = 1
    return t


def host_params(tree):
    c = tree.children
    L = len(c) // 2
    return ([c[f"w{i}"].value.numpy() for i in range(1, L + 1)],
            [c[f"b{i}"].value.numpy() for i in range(1, L + 1)])


def relu_masks(J, params, x_dev, xh, act):
    """Device sign patterns of the hidden pre-activations, after checking
    every element where they disagree with the oracle's is a near-tie:
    |z| within the reduction tolerance of 0 (relu' is discontinuous there and
    either branch is a correct rounding of the reference's arithmetic)."""
    if act != "relu":
        return None
    c = params.children
    L = len(c) // 2
    ws, bs = host_params(params)
    z_ref = orc.mlp_hidden_preacts(ws, bs, xh, act, threads=8)
    a = x_dev
    masks = []
    for i in range(1, L):
        z = a.dot(c[f"w{i}"].value.to(a.device())).add(c[f"b{i}"].value.to(a.device()))
        a = z.relu()
        zg = z.numpy()
        zr = z_ref[i - 1]
        m = zg > 0
        dis = m != (zr > 0)
        rms = float(np.sqrt(np.mean(zr.astype(np.float64) ** 2)))
        assert np.all(np.abs(zr[dis]) <= TOL_REDUCTION * rms), "relu sign flip away from a tie"
        masks.append(m)
    return masks


@pytest.mark.parametrize("dims,act,B,D", [([784, 512, 10], "tanh", 64, 2),
                                          ([256, 512, 512, 512, 100], "relu", 96, 2),
                                          ([1024, 4096, 4096, 4096, 1000], "relu", 64, 1)])
def test_dp_grad_step_matches_oracle(J, dims, act, B, D):
    """pmap-of-valueAndGradTree with psum-averaged grads (configs 0 and 4 shape)."""
    params = make_mlp(J, dims, 3)
    x = J.Random.normal(J.PRNGKey.key(1), J.Shape(D, B, dims[0]))
    labels = (orc.uniform(J.PRNGKey.key(2).state(), (D * B,)) * dims[-1]).astype(np.int64)
    t_host = onehot(labels, dims[-1]).reshape(D, B, dims[-1])
    t = J.ConcreteNDArray.of(t_host)
    devices = [J.Device(None) for _ in range(D)]
    loss = mlp_loss(J, act)
    Dn = J.ConcreteNDArray.scalar(float(D))
    out = {}

    def body(xs, ts):
        ploc = J.PyTrees.map(lambda a: a.to(xs.device()), params)
        v, g = J.JAX.valueAndGradTree(lambda p: loss(p, xs, ts))(ploc)
        g = J.Lax.psumTree(g)
        out[id(xs.device())] = J.PyTrees.map(lambda a: a.div(Dn.to(a.device())), g)
        return v

    losses = J.JAX.pmap(body, devices)(x, t).toFloatArray()
    ws, bs = host_params(params)
    xh = x.numpy()
    shards = [J.ConcreteNDArray.of(xh[i]) for i in range(D)]
    per = [orc.mlp_loss_grad(ws, bs, xh[i], t_host[i], act=act, threads=8,
                             relu_masks=relu_masks(J, params, shards[i], xh[i], act)) for i in range(D)]
    for i in range(D):
        assert abs(losses[i] - per[i][0]) <= TOL_REDUCTION * abs(per[i][0])
    g = next(iter(out.values())).children
    L = len(ws)
    for l in range(L):
        ref_w = orc.binary(orc.DIV, orc.psum([per[i][1][l] for i in range(D)]), np.float32([D]))
        ref_b = orc.binary(orc.DIV, orc.psum([per[i][2][l] for i in range(D)]), np.float32([D]))
        assert_rel(g[f"w{l + 1}"].value.numpy(), ref_w, TOL_REDUCTION, f"dW{l + 1}")
        assert_rel(g[f"b{l + 1}"].value.numpy(), ref_b, TOL_REDUCTION, f"db{l + 1}")


def test_grad_of_pmap_wrt_input(J):
    """JAX.grad(x -> pmap(loss(params, .)).sum()) -- the PMAP VJP path."""
    dims = [784, 512, 10]
    params = make_mlp(J, dims, 0)
    B, D = 32, 2
    x = J.Random.normal(J.PRNGKey.key(0), J.Shape(D, B, dims[0]))
    labels = (orc.uniform(7, (D * B,)) * 10).astype(np.int64)
    t_host = onehot(labels, 10)
    t_dev = [J.ConcreteNDArray.of(t_host[i * B:(i + 1) * B]) for i in range(D)]
    devices = [J.Device(None) for _ in range(D)]
    loss = mlp_loss(J, "tanh")
    # each shard's labels selected by its position: a 2-input pmap body
    t = J.ConcreteNDArray.of(t_host.reshape(D, B, 10))

    def f(xx):
        return J.JAX.pmap(lambda xs, ts: loss(params, xs, ts), devices)(xx, t).sum()

    gx = J.JAX.grad(f)(x).numpy()
    ws, bs = host_params(params)
    xh = x.numpy()
    for i in range(D):
        _, _, _, ref_gx = orc.mlp_loss_grad(ws, bs, xh[i], t_host[i * B:(i + 1) * B], act="tanh",
                                            want_gx=True, threads=8)
        assert_rel(gx[i], ref_gx, TOL_REDUCTION, f"gx shard {i}")


@pytest.mark.parametrize("rows,cols", [(8, 16384), (33, 1000), (4, 7)])
def test_elementwise_sweep(J, rows, cols):
    x = J.Random.normal(J.PRNGKey.key(1), J.Shape(rows, cols))
    y = J.Random.uniform(J.PRNGKey.key(11), J.Shape(rows, cols), -3.0, 3.0)
    zero = J.ConcreteNDArray.scalar(0.0)
    lo, hi = J.ConcreteNDArray.scalar(-1.0), J.ConcreteNDArray.scalar(1.0)
    z = J.Numpy.where(x.gt(zero), x.tanh().mul(y.sigmoid()), y.relu().clip(lo, hi))
    s = z.sum(-1, True)
    am = z.argmax(-1)
    rz, rs, ram = orc.sweep(x.numpy(), y.numpy(), want_z=True)
    assert_rel(z.numpy(), rz, TOL_ELEMENTWISE, "z")
    assert_rel(s.numpy(), rs, TOL_REDUCTION, "row sums")
    np.testing.assert_array_equal(am.numpy(), ram)


def test_config2_pmap_dot_allgather_full_size(J):
    """Config 2 at full size: two shards of A [4096,8192] (U(-1,1), seed 2)
    times a replicated B [8192,4096], gathered with Lax.allGather.  The
    oracle recomputes sampled rows of every shard (a full FP32 host dot of
    this size takes minutes); the rest is checked through a size-independent
    identity: (A_i . B) . 1 = A_i . (B . 1) on every row."""
    M, K, N, D = 4096, 8192, 4096, 2
    devices = [J.Device(None) for _ in range(D)]
    A = J.Random.uniform(J.PRNGKey.key(2), J.Shape(D, M, K), -1.0, 1.0)
    B = J.Random.uniform(J.Random.split(J.PRNGKey.key(2), 2)[1], J.Shape(K, N), -1.0, 1.0)
    out = J.JAX.pmap(lambda a: J.Lax.allGather(a.dot(B), D), devices)(A)
    assert out.shape().dimensions() == (D, D, M, N)
    c = out.numpy()
    np.testing.assert_array_equal(c[0], c[1])  # every shard holds the same gather
    ah, bh = A.numpy(), B.numpy()
    for i in range(D):
        for r0 in (0, 1733, M - 8):
            ref = orc.dot(ah[i], bh, rows=(r0, r0 + 8), threads=8)
            assert_rel(c[0, i, r0:r0 + 8], ref, TOL_REDUCTION, f"shard {i} rows {r0}..")
    ones = np.ones(N, np.float64)
    b1 = bh.astype(np.float64) @ ones
    for i in range(D):
        lhs = c[0, i].astype(np.float64) @ ones
        rhs = ah[i].astype(np.float64) @ b1
        assert_rel(lhs, rhs, TOL_REDUCTION, f"row-sum identity, shard {i}")


@pytest.mark.parametrize("mode,factor", [("slice", 1.0), ("reduce_scatter", 2.0)])
def test_all_gather_vjp_modes(J, mode, factor):
    """L = sum over 2 shards of sum(allGather(x) * c): dL/dx = 2c.  The
    reference's VJP (the local slice, Grad.java:437-441) gives c; the
    reduce-scatter VJP gives the true 2c."""
    from jax4j_b200 import pmap as P
    c = np.float32([[1, 2, 3], [4, 5, 6]])
    cc = J.ConcreteNDArray.of(c)
    x = J.ConcreteNDArray.of(np.float32([[0.5, -1, 2], [3, 0.25, -4]]))
    devices = [J.Device(None), J.Device(None)]
    old = P.ALLGATHER_VJP
    try:
        J.Lax.setAllGatherVjp(mode)
        fn = lambda v: J.JAX.pmap(lambda s: J.Lax.allGather(s, 2).mul(cc).sum(), devices)(v).sum()
        g = J.JAX.grad(fn)(x).numpy()
    finally:
        P.ALLGATHER_VJP = old
    np.testing.assert_allclose(g, factor * c, rtol=1e-6)


def test_headline_grad_step_full_batch_8192(J):
    """Config 4 at the size the benchmark times: one data-parallel grad step
    of the 1024-4096-4096-4096-1000 relu MLP at batch 8192 on one GPU, with
    the benchmark's seeds (Glorot weights from key 3, x ~ N(0,1) from key 1,
    labels from key 2).  The loss, every bias gradient and every weight
    gradient in full against the oracle's restatement of the reference's
    host step (all host threads; about a minute of CPU), and against an FP64
    computation of the same step."""
    import torch
    dims, B, D = [1024, 4096, 4096, 4096, 1000], 8192, 1
    params = make_mlp(J, dims, 3)
    x = J.Random.normal(J.PRNGKey.key(1), J.Shape(D, B, dims[0]))
    u = J.Random.uniform(J.PRNGKey.key(2), J.Shape(D * B))
    labels = np.minimum((u.numpy() * dims[-1]).astype(np.int64), dims[-1] - 1)
    t_host = onehot(labels, dims[-1]).reshape(D, B, dims[-1])
    t = J.ConcreteNDArray.of(t_host)
    loss = mlp_loss(J, "relu")
    out = {}

    def body(xs, ts):
        v, g = J.JAX.valueAndGradTree(lambda p: loss(p, xs, ts))(params)
        out["g"] = J.Lax.psumTree(g)
        return v

    losses = J.JAX.pmap(body, [J.Device.defaultDevice()])(x, t).toFloatArray()
    torch.cuda.synchronize()
    ws, bs = host_params(params)
    xh = x.numpy()[0]
    masks = relu_masks(J, params, J.ConcreteNDArray.of(xh), xh, "relu")
    ref_loss, ref_gw, ref_gb, _ = orc.mlp_loss_grad(ws, bs, xh, t_host[0], act="relu", threads=orc.nproc(),
                                                    relu_masks=masks)
    assert abs(losses[0] - ref_loss) <= TOL_REDUCTION * abs(ref_loss), (losses[0], ref_loss)
    g = out["g"].children
    exact_w, exact_b = _mlp_grads_fp64(ws, bs, xh, t_host[0], masks)
    for l in range(len(ws)):
        _assert_grad(g[f"b{l + 1}"].value.numpy(), ref_gb[l], exact_b[l], f"db{l + 1}")
        _assert_grad(g[f"w{l + 1}"].value.numpy(), ref_gw[l], exact_w[l], f"dW{l + 1}")


def _mlp_grads_fp64(ws, bs, x, onehot_t, masks):
    """The relu MLP's softmax cross-entropy gradients in FP64 (numpy), with
    the given relu masks: the exact values the FP32 computations round."""
    W = [w.astype(np.float64) for w in ws]
    acts, a = [], x.astype(np.float64)
    for l in range(len(W) - 1):
        acts.append(a)
        a = (a @ W[l] + bs[l]) * masks[l]
    acts.append(a)
    logits = a @ W[-1] + bs[-1]
    e = np.exp(logits)
    g = (e / e.sum(-1, keepdims=True) - onehot_t) / x.shape[0]
    gw, gb = [None] * len(W), [None] * len(W)
    for l in range(len(W) - 1, -1, -1):
        gw[l] = acts[l].T @ g
        gb[l] = g.sum(0)
        if l:
            g = (g @ W[l].T) * masks[l - 1]
    return gw, gb


def _assert_grad(got, ref, exact, what):
    """The device gradient against the oracle's at the reductions tolerance
    (per tensor) on all but at most one element in a million -- at a batch
    of 8192 the reference's own sequential FP32 sums carry errors of the
    order of the tolerance on a few elements of heavy cancellation -- and
    the device's worst error against the exact (FP64) gradient within 4
    times the reference's own worst error, or 10 times inside the tolerance,
    both relative to the gradient's rms."""
    got, ref, exact = (np.asarray(v, np.float64) for v in (got, ref, exact))
    rms = float(np.sqrt(np.mean(ref * ref)))
    beyond = np.abs(got - ref) > TOL_REDUCTION * np.maximum(np.abs(ref), rms)
    assert beyond.sum() <= max(1, got.size // 1_000_000), (what, int(beyond.sum()))
    e_dev = float(np.max(np.abs(got - exact))) / rms
    e_ref = float(np.max(np.abs(ref - exact))) / rms
    assert e_dev <= max(4 * e_ref, TOL_REDUCTION / 10), (what, e_dev, e_ref)


def _config0_inputs(J):
    """Config 0 exactly as the benchmark builds it: W1 [784,512], W2 [512,10]
    Glorot from keys split from key 0, zero biases, x [2,256,784] ~ N(0,1)
    from key 0, labels (int)(u * 10) from the third split key."""
    keys = J.Random.split(J.PRNGKey.key(0), 3)
    params = {"w1": J.Random.glorotUniform(keys[0], J.Shape(784, 512), 784, 512),
              "b1": J.ConcreteNDArray.full(J.Shape(512), 0.0),
              "w2": J.Random.glorotUniform(keys[1], J.Shape(512, 10), 512, 10),
              "b2": J.ConcreteNDArray.full(J.Shape(10), 0.0)}
    x = J.Random.normal(J.PRNGKey.key(0), J.Shape(2, 256, 784))
    labels = np.minimum((J.Random.uniform(keys[2], J.Shape(512)).numpy() * 10).astype(np.int64), 9)
    t_host = onehot(labels, 10).reshape(2, 256, 10)
    return params, x, t_host


def test_config0_full_size_both_parts(J):
    """Config 0 at its full size, x [2,256,784] over two pmap shards on one
    GPU: (i) the gradient of pmap(loss).sum() w.r.t. x, per shard; (ii) pmap
    of gradTree over {W1,b1,W2,b2} with psumTree -- against the oracle."""
    params, x, t_host = _config0_inputs(J)
    t = J.ConcreteNDArray.of(t_host)
    devices = [J.Device.defaultDevice(), J.Device(None, "shard1")]
    neg = J.ConcreteNDArray.scalar(-1.0)

    def loss_fn(p, xs, ts):
        h = xs.dot(p["w1"]).add(p["b1"]).tanh()
        logits = h.dot(p["w2"]).add(p["b2"])
        return J.Nn.softmax(logits).log().mul(ts).sum(-1).mean().mul(neg)

    gx = J.JAX.grad(lambda xx: J.JAX.pmap(lambda xs, ts: loss_fn(params, xs, ts), devices)(xx, t).sum())(x)
    out = {}

    def body(xs, ts):
        v, g = J.JAX.valueAndGradTree(
            lambda tr: loss_fn({k: tr.children[k].value for k in params}, xs, ts))(J.PyTree.dictOf(params))
        out[id(xs.device())] = J.Lax.psumTree(g)
        return v

    losses = J.JAX.pmap(body, devices)(x, t).toFloatArray()
    ws = [params["w1"].numpy(), params["w2"].numpy()]
    bs = [params["b1"].numpy(), params["b2"].numpy()]
    xh = x.numpy()
    per = [orc.mlp_loss_grad(ws, bs, xh[i], t_host[i], act="tanh", want_gx=True, threads=orc.nproc())
           for i in range(2)]
    gxh = gx.numpy()
    for i in range(2):
        assert abs(losses[i] - per[i][0]) <= TOL_REDUCTION * abs(per[i][0])
        assert_rel(gxh[i], per[i][3], TOL_REDUCTION, f"(i) dL/dx shard {i}")
    for g in out.values():  # every shard holds the same psum
        c = g.children
        for l, k in enumerate(("w1", "w2")):
            assert_rel(c[k].value.numpy(), orc.psum([per[0][1][l], per[1][1][l]]), TOL_REDUCTION, f"(ii) d{k}")
        for l, k in enumerate(("b1", "b2")):
            assert_rel(c[k].value.numpy(), orc.psum([per[0][2][l], per[1][2][l]]), TOL_REDUCTION, f"(ii) d{k}")
