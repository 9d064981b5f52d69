"""One rank of a tensor-parallel decode, run as its own process by
test_gpu_tp.py: loads its shard of the GGUF model on GPU `rank`, decodes
greedily and saves its tokens and its slice of every step's logits.

usage: tp_worker.py RANK WORLD MODEL ID_HEX PROMPT(comma-separated) N_NEW OUT.npz [P2P_DIR]

With P2P_DIR, the sessions' all-reduces run over NVLink peer memory
(Session.tp_attach); the ranks swap their handles as files in P2P_DIR.
"""
import os
import sys
import time

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def file_allgather(d, tag, rank, world, timeout=120.0):
    """allgather(bytes) over files in d: write this rank's, wait for all."""
    def gather(data):
        tmp = os.path.join(d, f"{tag}.{rank}.tmp")
        with open(tmp, "wb") as f:
            f.write(data)
        os.replace(tmp, os.path.join(d, f"{tag}.{rank}.bin"))
        names = [os.path.join(d, f"{tag}.{r}.bin") for r in range(world)]
        t0 = time.monotonic()
        while not all(os.path.exists(n) for n in names):
            if time.monotonic() - t0 > timeout:
                raise TimeoutError(f"rank {rank}: handles of {tag} missing")
            time.sleep(0.01)
        out = []
        for n in names:
            with open(n, "rb") as f:
                out.append(f.read())
        return out
    return gather


def main(argv):
    rank, world = int(argv[1]), int(argv[2])
    path, uid = argv[3], bytes.fromhex(argv[4])
    prompt = np.array([int(t) for t in argv[5].split(",")], np.uint32)
    n_new, out = int(argv[6]), argv[7]
    from chat_wgpu_b200.context import GpuContext
    from chat_wgpu_b200.model import Model, Session
    ctx = GpuContext(rank)
    m = Model(ctx, path, tp=(rank, world, uid))
    p2p = argv[8] if len(argv) > 8 else None
    s = Session(m, len(prompt) + n_new)
    assert not s.persistent
    if p2p:
        s.tp_attach_p2p(file_allgather(p2p, "s", rank, world))
    s.begin(prompt)
    s.run(len(prompt) - 1)
    logits = []
    for _ in range(n_new):
        s.run(1)
        logits.append(s.logits())
    toks = s.tokens()
    # what a tensor-parallel model does not support fails cleanly (no collective runs)
    from chat_wgpu_b200 import CwError
    t = Session(m, 16)
    t.begin(prompt[:4])
    for call in (lambda: t.set_sampling(0.8), t.prefill, lambda: t.add_tap("q", 0, 4)):
        try:
            call()
        except CwError:
            continue
        raise AssertionError("expected CwError")
    t.set_sampling(0.0)  # greedy stays available
    t.close()
    # a stop token (greedy): the stream ends before it, on every rank
    e = Session(m, len(prompt) + n_new)
    if p2p:
        e.tp_attach_p2p(file_allgather(p2p, "e", rank, world))
    e.set_eos([int(toks[3])])
    e.begin(prompt)
    e.run(len(prompt) - 1 + n_new)
    eos_toks, eos_stopped = e.tokens(), e.stopped
    e.close()
    np.savez(out, toks=toks, logits=np.stack(logits), vocab_offset=m.vocab_offset,
             vocab=m.vocab_size, weight_bytes=m.info["weight_bytes"], eos_toks=eos_toks,
             eos_stopped=eos_stopped)
    s.close()
    m.close()
    ctx.close()


if __name__ == "__main__":
    main(sys.argv)
