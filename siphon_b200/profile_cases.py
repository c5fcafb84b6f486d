"""Single-process workloads the committed ncu summaries (profiles/*.md) were
captured on, runnable under `ncu` on one GPU:

    python -m siphon_b200.profile_cases flat      # gemv_flat_kernel<Q4_K>, 4 x 27648x5120
    python -m siphon_b200.profile_cases ar        # gemv_kernel<Q4_K, AR> beside the plain one, 5120x13824
    python -m siphon_b200.profile_cases prefill   # prefill_kernel<Q4_K>, 4096x4096, 512 tokens
    python -m siphon_b200.profile_cases steps     # Wq/Wk/Wv of the 32B shape (5120 -> 5120+1024+1024,
                                                  # Q4_K) with the residual add + RMS norm fused,
                                                  # beside the same launch without the step
    python -m siphon_b200.profile_cases decode_full  # three eager decode steps of the TinyLlama-1.1B
                                                  # shape with the steps and attention, the token at
                                                  # position 511 of a 512-position context

Each case runs a few launches (the summaries' `-s` skips the first ones) and
exits non-zero if the library reports a device-side status bit.
"""

from __future__ import annotations

import sys


def main(case: str, reps: int = 4) -> int:
    import torch

    from . import lib, synth
    from . import quant as Q
    from .model_path import device_weights

    torch.cuda.set_device(0)
    s = lib.load()
    s.init(0)
    s.set_overlap(True)
    dev = torch.device("cuda", 0)
    if case == "flat":
        wt, n_out, n_in, c = Q.Q4_K, 27648, 5120, 4
        ws = [device_weights(wt, n_out, n_in, seed=1 + i, device=dev) for i in range(c)]
        x = torch.from_numpy(synth.activations(n_in, 1, seed=2)[0]).to(dev)
        ys = [torch.empty(n_out, device=dev) for _ in range(c)]
        for _ in range(reps):
            s.gemv_multi(wt, ws, [n_out] * c, n_in, x, ys)
    elif case == "ar":
        wt, n_out, n_in = Q.Q4_K, 5120, 13824
        g = s.ar_create(1, 0, n_out)
        g.open([g.local_handle])
        w = device_weights(wt, n_out, n_in, seed=1, device=dev)
        x = torch.from_numpy(synth.activations(n_in, 1, seed=2)[0]).to(dev)
        y = torch.empty(n_out, device=dev)
        for _ in range(reps):
            s.gemv_ar(wt, w, n_in, n_out, x, y, g)
            s.gemv_f32(wt, w, n_in, n_out, x, y)
        torch.cuda.synchronize()
        g.destroy()
    elif case == "prefill":
        wt, n, m = Q.Q4_K, 4096, 512
        w = device_weights(wt, n, n, seed=1, device=dev)
        x = torch.randn(m, n, device=dev)
        y = torch.empty(m, n, device=dev)
        for _ in range(2):
            s.gemm_prefill_f32(wt, w, n, n, x, m, y)
    elif case == "steps":
        wt, n_in, outs = Q.Q4_K, 5120, [5120, 1024, 1024]
        ws = [device_weights(wt, n, n_in, seed=1 + i, device=dev) for i, n in enumerate(outs)]
        x = torch.randn(n_in, device=dev)
        r = torch.randn(n_in, device=dev)
        gam = 1.0 + 0.1 * torch.randn(n_in, device=dev)
        h = torch.empty(n_in, device=dev)
        ys = [torch.empty(n, device=dev) for n in outs]
        for _ in range(reps):
            s.gemv_multi(wt, ws, outs, n_in, x, ys)
            s.gemv_fused(wt, ws, outs, n_in, x, lib.rms_norm_step(gam, 1e-6, r, h), ys)
    elif case == "decode_full":
        from . import model_path as mp
        from . import synth_model as sm
        m = mp.MatrixPath(s, sm.TINYLLAMA, dev, seed=4, attention=True, n_ctx=512)
        m.pos = 511
        st = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(st):
            for _ in range(3):
                m.decode_step(st)
        torch.cuda.synchronize()
        m.close()
    else:
        raise SystemExit(f"unknown case {case!r} (flat, ar, prefill, steps, decode_full)")
    torch.cuda.synchronize()
    st = s.status()
    print(case, "status", st)
    return 1 if st else 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1] if len(sys.argv) > 1 else "flat"))
