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
    elif args.scenario == "psum_sgd":
        # Lax.psumSgdTree's fused path (peer memory) against psumTree + the
        # elementwise update, over three steps; leaves sized to make several
        # buckets, one of them cut by the 16-segment limit
        import torch
        from jax4j_b200 import api as A, psum_sgd
        assert psum_sgd.ENABLED, "run with J4C_PSUM_SGD=1"
        old_bucket = A.PSUM_BUCKET_BYTES
        A.PSUM_BUCKET_BYTES = 1 << 20
        r = np.random.default_rng(100 + rank)
        shapes = [(512, 384), (384,), (384, 260), (260,)] + [(4 * (k + 1),) for k in range(18)] + [(1024, 300)]
        base = np.random.default_rng(7)
        params = J.PyTree.list(*[J.PyTree.leaf(J.ConcreteNDArray.of(base.standard_normal(s).astype(np.float32)))
                                 for s in shapes])
        scale, lr = 1.0 / D, 0.05
        p_fused, p_ref = params, params
        for step in range(3):
            grads = J.PyTree.list(*[J.PyTree.leaf(J.ConcreteNDArray.of(r.standard_normal(s).astype(np.float32)))
                                    for s in shapes])
            res = {}

            def fused_body(dummy):
                res["fused"] = J.Lax.psumSgdTree(p_fused, grads, scale, lr)
                return dummy

            def ref_body(dummy):
                g = J.Lax.psumTree(grads)
                upd = A._sgd_update(scale, lr)
                res["ref"] = J.PyTrees.unflatten(p_ref, [upd(w, gg) for w, gg in zip(J.PyTrees.flatten(p_ref),
                                                                                    J.PyTrees.flatten(g))])
                return dummy

            one = J.LocalShard(J.ConcreteNDArray.of(np.zeros(4, np.float32)), D)
            J.JAX.pmap(fused_body, devices)(one)
            J.JAX.pmap(ref_body, devices)(one)
            p_fused, p_ref = res["fused"], res["ref"]
        torch.cuda.synchronize()
        fl = [x.numpy() for x in J.PyTrees.flatten(p_fused)]
        rl = [x.numpy() for x in J.PyTrees.flatten(p_ref)]
        import ctypes as C
        from jax4j_b200 import _lib
        code = C.c_int(0)
        _lib.lib().j4c_device_status(C.byref(code))
        np.savez(args.out + f".rank{rank}", status=code.value, **{f"f{i}": a for i, a in enumerate(fl)},
                 **{f"r{i}": a for i, a in enumerate(rl)})
        A.PSUM_BUCKET_BYTES = old_bucket
    elif args.scenario == "psum_sgd_timeout":
        # rank 0 runs the fused update alone with a 1 ms wait limit: its waits
        # on rank 1's flags (which nothing sets) run out, the kernels record
        # status 0x7C05 and return; rank 1 stays alive (its buffer stays
        # mapped) and joins the host barrier afterwards
        import ctypes as C
        import torch
        from jax4j_b200 import _lib, psum_sgd
        shapes = [(256, 64), (64,)]
        w = [J.ConcreteNDArray.of(np.ones(s, np.float32)) for s in shapes]
        g = [J.ConcreteNDArray.of(np.ones(s, np.float32)) for s in shapes]
        psum_sgd._plan_for(st, tuple(x.shape().size() for x in w), 1 << 30)  # both ranks map the buffers
        distributed.barrier()
        if rank == 0:
            prev = C.c_uint64(0)
            _lib.lib().j4c_set_wait_limit_ns(1000000, C.byref(prev))
            from jax4j_b200 import api as A
            ctx_stream = A._comm_stream(w[0].tensor().device)
            out = psum_sgd.fused(None, st, w, g, 0.5, 0.1, ctx_stream, 1 << 30)
            torch.cuda.synchronize()
            _lib.lib().j4c_set_wait_limit_ns(prev.value, None)
            code = C.c_int(0)
            _lib.lib().j4c_device_status(C.byref(code))
            with open(args.out, "w") as f:
                f.write(str(code.value))
        distributed.barrier()
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
