"""Run CoRoPE forward + backward on one synthetic case (for ncu captures).

    python corope-jcx_b200/profile_case.py B H S D [steps] [algo]

bf16 N(0,1) inputs on cuda:0, theta 1e4, sm_scale 1/sqrt(D).  Prints "ok".
"""
import math
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import torch  # noqa: E402

from CoROPE.co_rope_backward import co_rope_backward  # noqa: E402
from CoROPE.forward import co_rope_forward  # noqa: E402


def main():
    B, H, S, D = (int(x) for x in sys.argv[1:5])
    steps = int(sys.argv[5]) if len(sys.argv) > 5 else 2
    algo = sys.argv[6] if len(sys.argv) > 6 else "auto"
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v, do = (torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16() for _ in range(4))
    sm = 1 / math.sqrt(D)
    for _ in range(steps):
        saved, _ = co_rope_forward(q, k, v, sm, algo=algo)
        co_rope_backward(saved, do, sm, algo=algo)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main()
