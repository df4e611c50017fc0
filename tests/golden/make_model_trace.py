"""Records the hot-path nodes of one real model run as fixtures.

    python tests/golden/make_model_trace.py [--reference /path/to/best-tts-godot]

Runs the reference's packed-model driver (tools/kpk_runtime.py:52-81,
``PackedModel.run`` over assets/model.kpk) on the reference's own sample
utterance (tools/voice_util.py ``sample_tokens(9)`` with the af_heart voice,
as kpk_runtime.py:84-95 does) and watches every ``RefRuntime.dispatch`` call
whose op is on the GPU path.  Runs in a container that has the reference
checkout; nothing else reads the reference.  Writes, next to this script:

  model_trace.npz  -- for a sample of those nodes, every input and output
                      array exactly as the reference produced it: for each op
                      type its smallest node plus up to five more nodes under
                      48 KB of traffic, spread over the graph;
  model_trace.json -- the sampled nodes (op, tensor ids, attributes as the
                      packed file stores them), the op counts of the whole
                      run, and every distinct node signature of the run:
                      op, attributes, and per input its dtype and shape, with
                      the values of inputs of at most 64 elements (axes,
                      shapes, split sizes, exponents, scalar constants),
                      and the number of outputs.
"""
import argparse
import collections
import json
import os
import sys
import warnings

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(REPO, "best-tts-godot_b200"))

import make_golden as G  # noqa: E402

SMALL_VALUES = 64          # inputs up to this many elements keep their values
SAMPLE_BYTES = 48 * 1024   # traffic bound of the extra sampled nodes
SAMPLE_EXTRA = 5


def spec(a):
    a = np.asarray(a)
    s = {"dtype": str(a.dtype), "shape": list(a.shape)}
    if a.size <= SMALL_VALUES:
        s["values"] = a.reshape(-1).tolist()
    return s


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("BT_REFERENCE_CHECKOUT"),
                    required="BT_REFERENCE_CHECKOUT" not in os.environ,
                    help="path of a best-tts-godot checkout (or set BT_REFERENCE_CHECKOUT)")
    args = ap.parse_args()
    ref_runtime, kpk_runtime = G.import_reference(args.reference)
    import voice_util
    from bt_b200.runtime import BtRuntime

    pm = kpk_runtime.PackedModel()
    ids = voice_util.sample_tokens(9)
    style = voice_util.load_voice("af_heart", len(ids))

    hot = []                        # (position, op, ins, outs, raw attrs, in arrays, out arrays, bytes)
    sigs = collections.OrderedDict()
    raw_attrs = {}
    for pos, (op_id, ins, outs, at, _place) in enumerate(pm.nodes):
        raw_attrs[(tuple(ins), tuple(outs))] = (pos, at or {})
    counts = collections.Counter()
    orig = ref_runtime.RefRuntime.dispatch

    def watch(self, op, node_input, node_output, at, env):
        if op not in BtRuntime.HOT_OPS:
            return orig(self, op, node_input, node_output, at, env)
        key = (tuple(int(i) if i else -1 for i in node_input), tuple(int(o) if o else -1 for o in node_output))
        pos, raw = raw_attrs[key]
        ins = [np.array(env[i], copy=True) if i else None for i in node_input]
        orig(self, op, node_input, node_output, at, env)
        outs = [np.array(env[o], copy=True) if o and o in env else None for o in node_output]
        nbytes = sum(a.nbytes for a in ins + outs if a is not None)
        counts[op] += 1
        hot.append((pos, op, list(node_input), list(node_output), raw, ins, outs, nbytes))
        sig = {"op": op, "attrs": raw, "inputs": [spec(a) if a is not None else None for a in ins],
               "n_out": len(node_output)}
        k = json.dumps(sig, sort_keys=True)
        if k in sigs:
            sigs[k]["count"] += 1
        else:
            sigs[k] = dict(sig, count=1, first=pos)

    ref_runtime.RefRuntime.dispatch = watch
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        wav = pm.run(ids, style)
    ref_runtime.RefRuntime.dispatch = orig

    by_op = collections.defaultdict(list)
    for h in hot:
        by_op[h[1]].append(h)
    picked = []
    for op, nodes in sorted(by_op.items()):
        chosen = {min(nodes, key=lambda h: h[7])[0]}
        small = [h for h in nodes if h[7] <= SAMPLE_BYTES and h[0] not in chosen]
        if small:
            step = max(1, len(small) // SAMPLE_EXTRA)
            chosen.update(h[0] for h in small[::step][:SAMPLE_EXTRA])
        picked += [h for h in nodes if h[0] in chosen]
    picked.sort(key=lambda h: h[0])

    arrays, sampled = {}, []
    for pos, op, ins, outs, raw, ia, oa, nbytes in picked:
        for j, a in enumerate(ia):
            if a is not None:
                arrays[f"n{pos}/in{j}"] = a
        for j, a in enumerate(oa):
            if a is not None:
                arrays[f"n{pos}/out{j}"] = a
        sampled.append({"pos": pos, "op": op, "inputs": ins, "outputs": outs, "attrs": raw, "bytes": nbytes})
    np.savez_compressed(os.path.join(HERE, "model_trace.npz"), **arrays)
    meta = {
        "source": "assets/model.kpk through tools/kpk_runtime.py PackedModel.run, sample_tokens(9), voice af_heart",
        "numpy": np.__version__,
        "nodes": len(pm.nodes),
        "hot_nodes": len(hot),
        "op_counts": dict(sorted(counts.items())),
        "waveform_samples": int(np.asarray(wav).size),
        "sampled": sampled,
        "signatures": list(sigs.values()),
    }
    with open(os.path.join(HERE, "model_trace.json"), "w") as f:
        json.dump(meta, f, separators=(",", ":"))
    print(f"{len(hot)} hot nodes of {len(pm.nodes)}, {len(sigs)} signatures, {len(sampled)} sampled nodes")


if __name__ == "__main__":
    main()
