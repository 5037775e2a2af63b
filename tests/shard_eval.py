"""Evaluates one rank's shard of a graph (ComputeGraph.shard(rank, world)) on
the host with the oracle's ops, f16 rounding after every operation as the
evaluator does; collectives are callables supplied by the test (gloo)."""
import numpy as np

import oracle


def evaluate_shard(desc, full_inputs, all_reduce, all_gather, threads=2):
    """desc: the shard description; full_inputs: graph value id -> whole
    array; all_reduce(x) -> sum over ranks; all_gather(x) -> list of every
    rank's x.  Returns {graph value id: array} for the shard's outputs."""
    q16 = oracle.quantize_f16
    values = desc["values"]
    vals = {}
    for v in values:
        if v["kind"] in (0, 1):
            x = q16(np.asarray(full_inputs[v["graph_value"]], dtype=np.float32))
            if v.get("slice") == "columns":
                x = x[..., v["range"][0]:v["range"][1]]
            elif v.get("slice") == "rows":
                x = x[..., v["range"][0]:v["range"][1], :]
            assert list(x.shape) == v["shape"], (x.shape, v)
            vals[v["id"]] = np.ascontiguousarray(x)
    for op in desc["ops"]:
        ins = [vals[i] for i in op["inputs"]]
        shape = values[op["result"]]["shape"]
        k = op["kind"]
        if k == "gemm":
            r = oracle.gemm(ins[0], ins[1], op["transpose_left"], op["transpose_right"])
        elif k == "gelu":
            r = oracle.gelu(ins[0])
        elif k == "add":
            r = ins[0] + ins[1]
        elif k == "split_heads":
            b, rows, w = ins[0].shape
            c = shape[2]
            r = ins[0].reshape(b, rows, w // c, c).transpose(0, 2, 1, 3).reshape(shape)
        elif k == "merge_heads":
            bh, rows, c = ins[0].shape
            h = shape[2] // c
            r = ins[0].reshape(bh // h, h, rows, c).transpose(0, 2, 1, 3).reshape(shape)
        elif k == "flash_attention":
            lead = ins[0].shape[:-2]
            s = int(np.prod(lead))
            r = oracle.attention(ins[0].reshape(s, *ins[0].shape[-2:]), ins[1].reshape(s, *ins[1].shape[-2:]),
                                 ins[2].reshape(s, *ins[2].shape[-2:]), scale=op["scale"] if op["scale"] > 0 else None,
                                 threads=threads).reshape(shape)
        elif k == "all_reduce":
            r = all_reduce(ins[0])
        elif k == "all_gather_columns":
            r = np.concatenate(all_gather(ins[0]), axis=-1)
        else:
            raise ValueError(k)
        assert list(r.shape) == shape, (k, r.shape, shape)
        vals[op["result"]] = q16(np.ascontiguousarray(r, dtype=np.float32))
    return {values[o]["graph_value"]: vals[o] for o in desc["outputs"]}
