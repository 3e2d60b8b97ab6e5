"""Worker for tests/test_gpu_multi.py, launched with torch.distributed.run
(one process per GPU).  Not collected by pytest."""
import argparse
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--scenario", required=True)
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    import jax4j_b200 as J
    from jax4j_b200 import distributed
    st = distributed.initialize(timeout_s=60.0)
    devices = distributed.global_devices()
    D, rank = st.world_size, st.rank
    if args.scenario == "dp_step":
        dims, B = [256, 512, 100], 64
        keys = J.Random.split(J.PRNGKey.key(3), 2)
        params = {"w1": J.Random.glorotUniform(keys[0], J.Shape(256, 512), 256, 512),
                  "b1": J.ConcreteNDArray.full(J.Shape(512), 0.0),
                  "w2": J.Random.glorotUniform(keys[1], J.Shape(512, 100), 512, 100),
                  "b2": J.ConcreteNDArray.full(J.Shape(100), 0.0)}
        x = J.Random.normal(J.PRNGKey.key(1), J.Shape(D * B, 256), offset=rank * B * 256,
                            count=B * 256).reshape(J.Shape(B, 256))
        lab = (np.arange(D * B) * 7919 % 100)[rank * B:(rank + 1) * B]
        t = np.zeros((B, 100), np.float32)
        t[np.arange(B), lab] = 1
        tt = J.ConcreteNDArray.of(t)
        neg = J.ConcreteNDArray.scalar(-1.0)

        def loss(p, xs, ts):
            c = p.children
            h = xs.dot(c["w1"].value).add(c["b1"].value).tanh()
            logits = h.dot(c["w2"].value).add(c["b2"].value)
            return J.Nn.softmax(logits).log().mul(ts).sum(-1).mean().mul(neg)

        out = {}

        def body(xs, ts):
            v, g = J.JAX.valueAndGradTree(lambda p: loss(p, xs, ts))(J.PyTree.dictOf(params))
            out["g"] = J.Lax.psumTree(g)
            return v

        losses = J.JAX.pmap(body, devices)(J.LocalShard(x, D), J.LocalShard(tt, D)).toFloatArray()
        if rank == 0:
            g = out["g"].children
            np.savez(args.out, losses=losses, x=np.concatenate([x.numpy()]), t=t,
                     **{k: params[k].numpy() for k in params},
                     **{"g_" + k: g[k].value.numpy() for k in params})
        else:
            np.savez(args.out + f".rank{rank}", x=x.numpy(), t=t)
    elif args.scenario == "grad_x":
        # grad of a pmap'd loss w.r.t. its sharded input, with LocalShard inputs
        keys = J.Random.split(J.PRNGKey.key(3), 2)
        params = {"w1": J.Random.glorotUniform(keys[0], J.Shape(64, 32), 64, 32),
                  "b1": J.ConcreteNDArray.full(J.Shape(32), 0.0),
                  "w2": J.Random.glorotUniform(keys[1], J.Shape(32, 10), 32, 10),
                  "b2": J.ConcreteNDArray.full(J.Shape(10), 0.0)}
        B = 16
        x = J.Random.normal(J.PRNGKey.key(1), J.Shape(D * B, 64), offset=rank * B * 64,
                            count=B * 64).reshape(J.Shape(B, 64))
        lab = (np.arange(D * B) * 31 % 10)[rank * B:(rank + 1) * B]
        t = np.zeros((B, 10), np.float32)
        t[np.arange(B), lab] = 1
        tt = J.ConcreteNDArray.of(t)
        neg = J.ConcreteNDArray.scalar(-1.0)

        def loss(xs, ts):
            h = xs.dot(params["w1"]).add(params["b1"]).tanh()
            logits = h.dot(params["w2"]).add(params["b2"])
            return J.Nn.softmax(logits).log().mul(ts).sum(-1).mean().mul(neg)

        tl = J.LocalShard(tt, D)
        gx = J.JAX.grad(lambda xx: J.JAX.pmap(loss, devices)(xx, tl).sum())(J.LocalShard(x, D))
        np.savez(args.out + f".rank{rank}", gx=gx.numpy(), x=x.numpy(), t=t,
                 **{k: params[k].numpy() for k in params})
    elif args.scenario == "leave":
        x = J.ConcreteNDArray.of(np.ones((D, 8), np.float32))
        J.JAX.pmap(lambda s: J.Lax.psum(s), devices)(x).toFloatArray()
        if rank == 1:
            os._exit(0)  # leaves between steps, nothing in flight
        try:
            J.JAX.pmap(lambda s: J.Lax.psum(s), devices)(x).toFloatArray()
            result = "no error"
        except J.CollectiveError as e:
            result = "CollectiveError: " + str(e)[:100]
        with open(args.out, "w") as f:
            f.write(result)
        os._exit(0)
    distributed.barrier()
    distributed.shutdown()


if __name__ == "__main__":
    main()
