"""Developer tool: launch timeline of the Llama-3.2-3B M=1 decode step (bench.py
``decode_gemv``) from a libqlinear built with -DQL_TRACE_TL.  For each of the four
GEMVs of a layer it prints the mean, over 10 CUDA-graph replays x 28 layers, of:
wait->end (work after griddepcontrol.wait), entry->wait (time a CTA sat resident before
its inputs were ready), prev_end->wait_min (release latency of the dependency),
entry_min-prev_end (negative: launched under the previous kernel) and the spread of
CTA end times (tail imbalance).  All from %globaltimer.

    cd mlx-gen_b200/csrc && nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
        -Xcompiler -fPIC -DQL_TRACE_TL -shared -o /tmp/tl/libqlinear.so libqlinear.cu
    QL_LIB_PATH=/tmp/tl/libqlinear.so python mlx-gen_b200/csrc/timeline.py
"""
import ctypes, os, sys
import numpy as np
_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if not os.environ.get("QL_LIB_PATH"):
    sys.exit("set QL_LIB_PATH to a libqlinear.so built with -DQL_TRACE_TL")
sys.path.insert(0, os.path.join(_ROOT, "mlx-gen_b200"))
sys.path.insert(0, _ROOT)
import torch, bench, qlinear
from qlinear import _lib
dev = torch.device("cuda:0")
r = bench.decode_gemv(dev, steps=10, warmup=3, head=False)
print({k: r[k] for k in ("value", "ms_per_step")})
torch.cuda.synchronize()
L = _lib.lib()
rec = np.dtype([("nentry_min", "u8"), ("entry_max", "u8"), ("nwait_min", "u8"), ("wait_max", "u8"),
                ("nend_min", "u8"), ("end_max", "u8"), ("kind", "u4"), ("grid", "u4"), ("done", "u4"), ("pad", "u4")])
buf = np.zeros(8192, rec)
cnt = ctypes.c_uint(0)
rc = L.ql_debug_timeline(ctypes.c_void_p(buf.ctypes.data), ctypes.c_size_t(buf.nbytes), ctypes.byref(cnt))
n = cnt.value
print("rc", rc, "launches", n)
b = buf[:n]
inv = lambda a: (~a.astype(np.uint64)).astype(np.int64)
e0, e1 = inv(b["nentry_min"]), b["entry_max"].astype(np.int64)
w0, w1 = inv(b["nwait_min"]), b["wait_max"].astype(np.int64)
d0, d1 = inv(b["nend_min"]), b["end_max"].astype(np.int64)
names = {2: "regs", 3: "regs-swiglu", 4: "tma", 5: "tma-swiglu"}
# last 10 replays x 112 launches
k = 112 * 10
sl = slice(n - k, n)
pos = np.arange(n)[sl] % 4
for p in range(4):
    idx = np.arange(n)[sl][pos == p]
    kinds = set(b["kind"][idx])
    post = (d1 - w0)[idx]
    pre = (w0 - e0)[idx]
    prev = idx - 1
    gap = (w0[idx] - d1[prev])
    ov = (e0[idx] - d1[prev])
    tail = (d1 - d0)[idx]
    wspread = (w1 - w0)[idx]
    print(f"pos {p} {[names.get(int(x)) for x in kinds]} grid {set(b['grid'][idx])}: "
          f"wait->end {post.mean()/1e3:.2f}us  entry->wait {pre.mean()/1e3:.2f}  prev_end->wait_min {gap.mean()/1e3:.2f}  "
          f"entry_min-prev_end {ov.mean()/1e3:.2f}  end spread {tail.mean()/1e3:.2f}  wait spread {wspread.mean()/1e3:.2f}")
per_layer = (d1[n - 1] - d1[n - 1 - 112 * 9]) / 9 / 28
print("per layer us", per_layer / 1e3)


