"""Per-phase timing of the persistent decode-step kernel (``sb_step_desc.trace``).

Runs one traced decode step of the synthetic decoder (engine ``"step"``) after
a prompt and reports, per layer (median over CTAs, microseconds), when each
operator boundary is reached, and for the middle layer the events of the
per-warp timeline (SM clock) that the kernel records - the ends of the four
projections, the attention item's milestones, the o_proj / down prologues and
the grid joins - as the time the last warp of a CTA reached each (median over
CTAs). The untraced step time (CUDA graph, CUDA events) is reported beside it.

    python -m spark_b200.steptrace [--layers 36] [--prompt 1024] [--json out.json]
"""

import argparse
import json

import numpy as np
import torch

from ._lib import lib
from .decoder import DecoderConfig, SyntheticDecoder

MARKS_PER_LAYER = 9
TIMELINE_EVENTS = 96  # per consumer warp
CONSUMER_WARPS = 11
PHASES = ["qkv_prologue", "qkv", "attention", "o_prologue", "o", "join_o", "gu_prologue", "gu", "down_prologue",
          "down", "join_down"]
PROJ_ENDS = ["qkv_end", "o_end", "gu_end", "down_end"]  # the four run_partials ends of a layer, in order
EVENTS = {1: "layer", 2: "fold", 3: "staged",
          20: "slice", 21: "item", 22: "q_built", 23: "computed", 24: "merged", 25: "published", 26: "qk_start",
          27: "qk_end", 28: "softmax_end", 30: "o_wait", 31: "o_ready", 32: "o_merged", 33: "o_staged",
          40: "join_enter", 41: "join_arrive", 42: "join_released", 43: "join_seen", 44: "join_exit",
          50: "gu_fold", 51: "gu_folded", 52: "gu_staged", 60: "down_wait", 61: "down_ready", 62: "down_staged"}


def _untraced_us(dec, reps=20):
    dec.capture()
    for _ in range(3):
        dec.graph.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        dec.graph.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / reps


def trace(dec):
    """One traced step of ``dec`` (engine "step"); returns the summary dict."""
    layers = dec.cfg.num_layers
    slots = lib().sb_step_trace_slots(layers)
    nsm = torch.cuda.get_device_properties(dec.device).multi_processor_count
    buf = torch.zeros(nsm * slots * 4, dtype=torch.int64, device=dec.device)
    dec.stepper.desc.trace = buf.data_ptr()
    try:
        for _ in range(2):
            buf.zero_()
            dec.step()
            torch.cuda.synchronize()
    finally:
        dec.stepper.desc.trace = None
    t = buf.view(nsm, slots, 4).cpu().numpy().astype(np.int64)
    nm = layers * MARKS_PER_LAYER
    start = t[:, nm + 1, 0].astype(np.float64)
    m0 = (t[:, :nm, 0] - start[:, None]) / 1000.0
    m1 = (t[:, :nm, 1] - start[:, None]) / 1000.0
    phases = {k: [] for k in PHASES}
    med = lambda a: float(np.median(a))  # noqa: E731
    for li in range(layers):
        b = li * MARKS_PER_LAYER
        prev = m1[:, b - 1] if li > 0 else np.zeros(nsm)
        phases["qkv_prologue"].append(med(m0[:, b] - prev))
        phases["qkv"].append(med(m0[:, b + 1] - m0[:, b]))
        phases["attention"].append(med(m0[:, b + 2] - m0[:, b + 1]))
        phases["o_prologue"].append(med(m0[:, b + 3] - m0[:, b + 2]))
        phases["o"].append(med(m0[:, b + 4] - m0[:, b + 3]))
        phases["join_o"].append(float(m1[:, b + 4].max() - m0[:, b + 4].max()))
        phases["gu_prologue"].append(med(m0[:, b + 5] - m1[:, b + 4]))
        phases["gu"].append(med(m0[:, b + 6] - m0[:, b + 5]))
        phases["down_prologue"].append(med(m0[:, b + 7] - m0[:, b + 6]))
        phases["down"].append(med(m0[:, b + 8] - m0[:, b + 7]))
        phases["join_down"].append(float(m1[:, b + 8].max() - m0[:, b + 8].max()))
    out = {"traced_step_us": float((t[:, nm, 0] - t[:, nm + 1, 0]).max() / 1000.0),
           "lm_head_us": med((t[:, nm, 0] - start) / 1000.0 - m1[:, nm - 1]),
           "per_layer_us": {k: round(float(np.mean(v)), 3) for k, v in phases.items()}}
    # the middle layer's per-warp timeline: per CTA the last warp to reach each event, median over CTAs
    tl0 = slots - CONSUMER_WARPS * TIMELINE_EVENTS // 2
    ev = t[:, tl0:, :].reshape(nsm, CONSUMER_WARPS, TIMELINE_EVENTS, 2)
    clk0 = t[:, nm + 1, 1].astype(np.float64)
    mid = layers // 2
    ghz = []
    firsts = {}
    for c in range(nsm):
        staged = [e for e in ev[c, 0] if int(e[0]) & 0xFFFFFFFF == 3 and e[1] != 0]
        if not staged:
            continue
        rate = (staged[0][1] - clk0[c]) / (t[c, mid * MARKS_PER_LAYER, 0] - start[c])  # cycles per ns
        ghz.append(rate)
        base = float(ev[c, 0, 0, 1])
        seen = {}  # event -> latest warp to reach it (the CTA's time for it)
        for w in range(CONSUMER_WARPS):
            ends = 0
            for code, clk in ev[c, w]:
                if clk == 0:
                    break
                code = int(code) & 0xFFFFFFFF
                if code == 15:
                    name = PROJ_ENDS[min(ends, 3)]
                    ends += 1
                else:
                    name = EVENTS.get(code)
                if name is None:
                    continue
                us = (float(clk) - base) / rate / 1000.0
                seen[name] = max(seen[name], us) if name in seen else us
        for k, v in seen.items():
            firsts.setdefault(k, []).append(v)
    out["middle_layer"] = mid
    order = sorted(firsts.items(), key=lambda kv: med(kv[1]))
    out["middle_layer_events_us"] = {k: round(med(v), 2) for k, v in order}
    out["sm_ghz"] = round(med(ghz), 3) if ghz else None
    return out


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--layers", type=int, default=36)
    p.add_argument("--prompt", type=int, default=1024)
    p.add_argument("--json", default=None, help="also write the summary here")
    args = p.parse_args(argv)
    cfg = DecoderConfig(num_layers=args.layers)
    dec = SyntheticDecoder(cfg, batch=1, capacity=args.prompt + 64, seed=0, engine="step")
    prompt = torch.randint(0, cfg.vocab, (1, args.prompt), generator=torch.Generator().manual_seed(0),
                           dtype=torch.int32).cuda()
    dec.prefill(prompt)
    torch.cuda.synchronize()
    summary = {"untraced_step_us": _untraced_us(dec)}
    summary.update(trace(dec))
    dec.check_status()
    text = json.dumps(summary, indent=1)
    print(text)
    if args.json:
        with open(args.json, "w") as f:
            f.write(text + "\n")


if __name__ == "__main__":
    main()
