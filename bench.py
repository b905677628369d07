#!/usr/bin/env python
"""Generator train-step throughput: audio-seconds trained per second.

Workload: the 40 kHz RVC v2 NSF-HiFiGAN generator training step (forward, backward with dL/dy
given, AdamW), batch 16 per GPU, 32 frames (12,800 samples) per item, 9-harmonic sine source,
cond(g), weight norm; forward GEMM operands as fp16 hi + scaled-lo pairs (three products,
fp32-accurate), backward operands bf16, fp32 accumulation.  AdamW at RVC's learning rate 1e-4.
Synthetic seeded inputs of the configured shapes (z ~ N(0,1), g ~ N(0,1), f0 ~ U(80,400) Hz with
20% unvoiced frames, dL/dy ~ N(0,1)).

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]

One process per GPU (torchrun for N > 1); gradients are all-reduced over NCCL inside the step.
Rank 0 prints one JSON line.  `--impl reference` times the reference's own CPU trainer
(src/wubu_train.c built from its sources into oracle/_ref) on this host's cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "generator train-step audio-sec/sec"
LR = 1e-4
UNIT = "audio-s/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="40k")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--frames", type=int, default=32)
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "fp32"],
                    help="backward GEMM arithmetic: bf16 operands, or fp32 (bf16 hi + lo pairs, three products)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only-device", action="store_true",
                    help="time only the device-resident steps (for profiler launch lists)")
    ap.add_argument("--infer", action="store_true",
                    help="forward-only long-clip inference (40 kHz, batch 1, 6000 frames = 2.4M samples, f0 "
                         "median-filtered over 5 frames) on one GPU: prints its own JSON line and exits")
    ap.add_argument("--gan", action="store_true",
                    help="the discriminator side of one RVC GAN iteration (MultiPeriodDiscriminator, periods "
                         "2..17, batch --batch of --frames x hop samples): discriminator step with AdamW, then "
                         "generator_loss + feature_loss and dL/dy_hat; prints its own JSON line and exits")
    ap.add_argument("--kernel", default=None, metavar="WHICH,STAGE",
                    help="time one convolution of the step alone (kernel_bench: which 0 f1, 1 d1, 2 g1, 3 f2, "
                         "4 d2, 5 ups forward, 6 ups input gradient, 7 ups weight gradient, 8 conv_pre, 9 g2) inside an NVTX range 'kb<which><stage>' and exit")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), d["hbm_gbs"], "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def make_inputs(cfg, B, F, seed):
    rng = np.random.default_rng(seed)
    T = F * int(np.prod(cfg["upsample_rates"]))
    z = rng.standard_normal((B, cfg["in_channels"], F), dtype=np.float32)
    g = rng.standard_normal((B, cfg["gin_channels"]), dtype=np.float32)
    f0 = rng.uniform(80, 400, (B, F)).astype(np.float32)
    f0[rng.random((B, F)) < 0.2] = 0.0
    dldy = rng.standard_normal((B, T), dtype=np.float32)
    return z, f0, g, dldy


class Clocks:
    """Samples SM clocks and throttle reasons of one GPU while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.f = None

    def __enter__(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.2)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.f:
            return None
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.f.name)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        load = [r[0] for r in rows]
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


def cpu_reference_step(ref, mel, dldy):
    ref.forward(mel)
    ref.backward(dldy)
    ref.adamw()


def time_reference(cfg_name, F, steps, warmup):
    """The reference C trainer (decoder fwd + bwd + AdamW, one item per step) on host cores."""
    from oracle import generator_ref as G
    from oracle import ref_oracle
    from wuburvc_b200 import model
    if not ref_oracle.available():
        return None, "oracle/_ref/libwubu_ref.so not built"
    cfg = model.decoder_only(cfg_name)
    P = G.init_params_ref(cfg, 1)
    ref = ref_oracle.RefTrainer(P, cfg["upsample_rates"], cfg["upsample_kernels"])
    T = F * model.hop(cfg)
    mel = G.counter_normal(1, 1, 192 * F).reshape(192, F).astype(np.float32)
    dldy = G.counter_normal(1, 2, T).astype(np.float32)
    for _ in range(warmup):
        cpu_reference_step(ref, mel, dldy)
    t0 = time.perf_counter()
    for _ in range(steps):
        cpu_reference_step(ref, mel, dldy)
    dt = (time.perf_counter() - t0) / steps
    audio_s = T / cfg["sr"]
    return {"value": audio_s / dt, "unit": UNIT, "cores": ref_oracle.RefTrainer.threads(), "kind": "reference",
            "sec_per_item": dt,
            "sample": f"1 item x {F} frames ({T} samples) per step, decoder fwd+bwd+AdamW of src/wubu_train.c "
                      f"(no NSF source / cond / noise convs: the reference trainer has none), {steps} steps"}, None


def run_reference(args, rank):
    if rank != 0:
        return
    res, why = time_reference(args.config, args.frames, args.steps, args.warmup)
    if res is None:
        print(json.dumps({"impl": "reference", "unavailable": why}))
        return
    ms = 1000.0 * res["sec_per_item"]
    # n_gpus: the N this arm was launched for (rank 0 alone runs the host trainer)
    line = {"impl": "reference", "metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": args.gpus,
            "host_only": True,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{args.config} generator train step on the reference CPU trainer, "
                                   f"1 item x {args.frames} frames per step (bounded sample of the batch-16 "
                                   f"workload)", "frames": args.frames, "parallelism": "OpenMP host threads"},
            "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the roofline kernel, from the ncu
# capture in profiles/tc_conv2_fwd_conv1_stage1_40k.md: 13.91 MB read + 512 B written at batch 8 (the
# output is still in L2 when the kernel ends), scaled by the rows to batch 16
TRAFFIC_BYTES = 2 * (13.913856e6 + 512)


def run_infer(args):
    """Forward-only inference of one long clip, inputs resident (value) and through the public API
    with the host inputs uploaded and the audio read back every call (e2e)."""
    import ctypes

    import torch
    from wuburvc_b200 import Generator, L, model

    cfg = model.config(args.config)
    B, F = 1, (args.frames if args.frames != 32 else 6000)
    gen = Generator(cfg, B, F, device=0)
    gen.set_forward_only(True)  # inference: nothing the backward would read is written
    z, f0, g, _ = make_inputs(cfg, B, F, seed=4321)
    # f0 smoothed with a 5-frame median filter (voiced frames only), 20 % unvoiced
    pad = np.pad(f0, ((0, 0), (2, 2)), mode="edge")
    med = np.median(np.stack([pad[:, i:i + F] for i in range(5)]), axis=0).astype(np.float32)
    f0 = np.where(f0 > 0, med, 0.0).astype(np.float32)
    gen.upload(z, f0, g, None, None)
    stream = torch.cuda.ExternalStream(gen.stream, device=0)
    fwd = L().wubu_b200_gen_forward
    audio = np.empty((B, gen.T), np.float32)

    def timed(fast):
        """(resident ms, e2e ms, audio) of one forward mode"""
        gen.set_forward_only(True, fast=fast)
        for _ in range(max(3, args.warmup)):
            check_rc(fwd(gen.h, 0, None))
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record(stream)
        for i in range(args.steps):
            check_rc(fwd(gen.h, i, None))
        e.record(stream)
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / args.steps
        s2, e2 = torch.cuda.Event(True), torch.cuda.Event(True)
        s2.record(stream)
        for i in range(args.steps):
            gen.upload(z, f0, g, None, None)
            check_rc(fwd(gen.h, i, audio.ctypes.data_as(ctypes.c_void_p)))
        e2.record(stream)
        torch.cuda.synchronize()
        assert np.isfinite(audio).all()
        return ms, s2.elapsed_time(e2) / args.steps, audio.copy()

    ms_x, ms_e2e_x, a_x = timed(False)  # exact: fp16 operand pairs
    ms, ms_e2e, a_f = timed(True)        # fast: single fp16 operands
    secs = B * gen.T / cfg["sr"]
    fl = 29.26e9 * (F / 32.0) * B  # algorithmic forward GFLOP per 32-frame item, scaled
    print(json.dumps({"metric": "generator forward (inference) audio-sec/sec", "value": secs / (ms / 1e3),
                      "unit": "audio-s/s", "n_gpus": 1, "steps": args.steps, "ms_per_step": ms,
                      "higher_is_better": True, "dtype": "fp16 operands, fp32 accumulate (fast inference)",
                      "data": "synthetic",
                      "config": {"workload": f"40 kHz long-clip inference, batch 1, {F} frames "
                                             f"({gen.T} samples), f0 median-filtered, 20% unvoiced"},
                      "e2e": {"value": secs / (ms_e2e / 1e3), "unit": "audio-s/s",
                              "h2d_bytes_per_step": int(z.nbytes + f0.nbytes + g.nbytes),
                              "d2h_bytes_per_step": int(audio.nbytes), "ms_per_step": ms_e2e},
                      "algorithmic_tflops": fl / (ms / 1e3) / 1e12,
                      "exact_pairs": {"value": secs / (ms_x / 1e3), "ms_per_step": ms_x,
                                      "e2e_value": secs / (ms_e2e_x / 1e3),
                                      "dtype": "fp16 operand pairs (3 products), fp32 accumulate"},
                      "fast_vs_exact_rel_l2": float(np.linalg.norm(a_f - a_x) / np.linalg.norm(a_x))}))
    gen.close()


def gan_flops(B, T, periods=(2, 3, 5, 7, 11, 17)):
    """Algorithmic FLOPs of one discriminator iteration: forward over real + generated twice (the
    discriminator step and the generator side), the weight gradients and the input gradients of
    every layer but the first in the discriminator step, and the input gradients of every layer
    over the generated half on the generator side."""
    s_layers = [(1, 16, 15, 1, 1, 7), (16, 64, 41, 4, 4, 20), (64, 256, 41, 4, 16, 20), (256, 1024, 41, 4, 64, 20),
                (1024, 1024, 41, 4, 256, 20), (1024, 1024, 5, 1, 1, 2), (1024, 1, 3, 1, 1, 1)]
    p_layers = [(1, 32, 5, 3, 1, 2), (32, 128, 5, 3, 1, 2), (128, 512, 5, 3, 1, 2), (512, 1024, 5, 3, 1, 2),
                (1024, 1024, 5, 1, 1, 2), (1024, 1, 3, 1, 1, 1)]
    total = 0.0
    for p in (0,) + tuple(periods):
        q = p or 1
        L, N = -(-T // q), 2 * B * q
        for li, (ci, co, k, st, grp, pad) in enumerate(p_layers if p else s_layers):
            L = (L + 2 * pad - k) // st + 1
            f = 2.0 * N * L * co * (ci // grp) * k  # one pass over both halves
            total += 2 * f + f + (f if li else 0) + f / 2
    return total


def run_gan(args):
    """The discriminator side of one GAN training iteration, inputs resident (value) and through the
    public API with host inputs and dL/dy_hat read back (e2e)."""
    import ctypes

    import torch
    from wuburvc_b200 import gan, model

    cfg = model.config(args.config)
    B, T = args.batch, args.frames * model.hop(cfg)
    rng = np.random.default_rng(77)
    flat = np.zeros(gan.param_total(), np.float32)
    for name, (off, shp) in gan.param_table().items():
        n = int(np.prod(shp))
        if name.endswith("weight_v"):
            v = rng.standard_normal(shp).astype(np.float32) / np.sqrt(shp[1] * shp[2])
            flat[off:off + n] = v.reshape(-1)
            flat[off - shp[0]:off] = np.sqrt((v.reshape(shp[0], -1) ** 2).sum(1))  # weight_g = ||v||
        elif name.endswith("bias"):
            flat[off:off + n] = 0.01 * rng.standard_normal(n)
    y = (0.3 * rng.standard_normal((B, T))).astype(np.float32)
    y_hat = (0.5 * y + 0.2 * rng.standard_normal((B, T))).astype(np.float32)
    d = gan.Discriminator(B, T)
    d.set_params(flat)
    Lh = gan.L()
    yd, yhd = torch.from_numpy(y).cuda(), torch.from_numpy(y_hat).cuda()
    dyd = torch.empty_like(yhd)
    stream = torch.cuda.ExternalStream(Lh.wubu_b200_disc_stream(d.h), device=0)
    torch.cuda.synchronize()

    def device_iter():
        check_rc(Lh.wubu_b200_disc_step(d.h, yd.data_ptr(), yhd.data_ptr(), gan.DEVICE, None))
        n = Lh.wubu_b200_disc_launches(d.h)
        check_rc(Lh.wubu_b200_disc_gen_loss(d.h, yd.data_ptr(), yhd.data_ptr(), dyd.data_ptr(), gan.DEVICE, None))
        return n + Lh.wubu_b200_disc_launches(d.h)

    for _ in range(max(3, args.warmup)):
        launches = device_iter()
    torch.cuda.synchronize()
    with Clocks(0) as clk:
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record(stream)
        for _ in range(args.steps):
            device_iter()
        e.record(stream)
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / args.steps
        # e2e: host waveforms in, dL/dy_hat and the losses out, every iteration
        dy = np.empty((B, T), np.float32)
        losses = np.zeros(2, np.float32)
        loss_d = np.zeros(1, np.float32)
        vp = ctypes.c_void_p
        s2, e2 = torch.cuda.Event(True), torch.cuda.Event(True)
        s2.record(stream)
        for _ in range(args.steps):
            check_rc(Lh.wubu_b200_disc_step(d.h, y.ctypes.data_as(vp), y_hat.ctypes.data_as(vp), 0,
                                            loss_d.ctypes.data_as(vp)))
            check_rc(Lh.wubu_b200_disc_gen_loss(d.h, y.ctypes.data_as(vp), y_hat.ctypes.data_as(vp),
                                                dy.ctypes.data_as(vp), 0, losses.ctypes.data_as(vp)))
        e2.record(stream)
        torch.cuda.synchronize()
        ms_e2e = s2.elapsed_time(e2) / args.steps
    assert np.isfinite(dy).all() and np.isfinite(losses).all() and np.isfinite(loss_d).all()
    clocks = clk.summary()
    secs = B * T / cfg["sr"]
    fl = gan_flops(B, T)
    mhz = (clocks or {}).get("sm_max_mhz") or 1965.0
    peak = 148 * 128 * 2 * mhz * 1e6 / 1e12  # fp32 FMA lanes x 2 FLOP x clock
    cpu = None
    if not args.no_cpu_baseline:
        import torch as th

        from oracle import gan_ref

        th.set_num_threads(os.cpu_count() or 1)
        P = gan_ref.init_params()
        t0 = time.time()
        gan_ref.d_step(P, y[:1], y_hat[:1], dtype=th.float32)
        gan_ref.g_step(P, y[:1], y_hat[:1], dtype=th.float32)
        dt = time.time() - t0
        cpu = {"value": (T / cfg["sr"]) / dt, "unit": "audio-s/s", "cores": th.get_num_threads(), "kind": "port",
               "sample": f"one item ({T} samples): upstream's discriminator step + generator side in torch "
                         f"float32 on the host cores (oracle/gan_ref.py), {dt:.2f} s"}
    print(json.dumps({"metric": "GAN discriminator iteration audio-sec/sec", "value": secs / (ms / 1e3),
                      "unit": "audio-s/s", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
                      "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                      "dtype": "fp32", "data": "synthetic",
                      "config": {"workload": f"MultiPeriodDiscriminator (S + periods 2,3,5,7,11,17), batch {B} x "
                                             f"{T} samples real + generated: discriminator step + AdamW, then "
                                             "generator_loss + feature_loss and dL/dy_hat",
                                 "l2": "activations ~1.4 GB per iteration, larger than L2"},
                      "e2e": {"value": secs / (ms_e2e / 1e3), "unit": "audio-s/s",
                              "h2d_bytes_per_step": int(4 * y.nbytes), "d2h_bytes_per_step": int(dy.nbytes + 12),
                              "ms_per_step": ms_e2e},
                      "gpu_launches": launches,
                      "roofline": {"bound": "fp32 FMA (CUDA cores)", "achieved": fl / (ms / 1e3) / 1e12,
                                   "peak": peak, "unit": "TFLOP/s", "frac": fl / (ms / 1e3) / 1e12 / peak,
                                   "peak_source": "nominal: 148 SMs x 128 fp32 lanes x 2 x sampled max clock",
                                   "traffic": None},
                      "cpu_baseline": cpu, "clocks": clocks}))
    d.close()


def check_rc(rc):
    if rc != 0:
        raise RuntimeError(f"wuburvc_b200 call failed ({rc})")


def main():
    args = parse()
    if args.infer:
        run_infer(args)
        return
    if args.gan:
        run_gan(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist
    from wuburvc_b200 import Generator, model

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=300))
    cfg = model.config(args.config)
    B, F = args.batch, args.frames
    # learning rate of RVC's own generator training (configs/v2/*.json "learning_rate": 1e-4)
    gen = Generator(cfg, B, F, device=local, lr=LR, precision=args.dtype)
    # Each timed phase starts from the initial parameters (which also restarts AdamW): AdamW on a
    # constant synthetic dL/dy drifts every weight the same way, and a few dozen steps later the
    # activations leave the fp16 range of the forward operands; the library would then switch the
    # context to bf16 operand pairs, and its one-time re-capture would land inside a timed region.
    p_init = gen.get_params()
    if world > 1:
        obj = [Generator.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        gen.attach_comm(rank, world, obj[0])
    T = gen.T
    z, f0, g, dldy = make_inputs(cfg, B, F, seed=1234 + rank)
    gen.upload(z, f0, g, None, dldy)
    stream = torch.cuda.ExternalStream(gen.stream, device=local)
    if args.kernel:  # one convolution alone (for a profiler capture)
        which, stage = (int(x) for x in args.kernel.split(","))
        gen.forward(0)
        gen.backward()
        gen.sync()
        torch.cuda.nvtx.range_push(f"kb{which}{stage}")
        kms, kflops = gen.kernel_bench(which, stage, iters=5)
        torch.cuda.nvtx.range_pop()
        print(json.dumps({"kernel": {"which": which, "stage": stage, "batch": B, "launch_ms": kms,
                                     "algorithmic_tflops": kflops / (kms / 1000.0) / 1e12}}))
        gen.close()
        return

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timing ----
    gen.set_params(p_init)
    for i in range(max(3, args.warmup)):
        gen.step_async(i)
    gen.sync()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(stream)
        for i in range(args.steps):
            gen.step_async(1000 + i)
        e1.record(stream)
        gen.sync()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    audio_s = B * T / cfg["sr"]
    value = world * audio_s / (ms / 1000.0)

    if args.only_device:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": value, "unit": UNIT, "ms_per_step": ms,
                              "gpu_launches": gen.graph_kernels() * args.steps, "note": "device-only run"}))
        gen.close()
        if world > 1:
            dist.destroy_process_group()
        return

    # ---- end to end through the public API: pinned host inputs in, audio out, every step ----
    gen.set_params(p_init)
    pz = torch.from_numpy(z).pin_memory()
    pf = torch.from_numpy(f0).pin_memory()
    pg = torch.from_numpy(g).pin_memory()
    pd = torch.from_numpy(dldy).pin_memory()
    pa = torch.empty((B, T), dtype=torch.float32).pin_memory()
    for i in range(2):
        gen.train_step_raw(pz.data_ptr(), pf.data_ptr(), pg.data_ptr(), pd.data_ptr(), pa.data_ptr(), i)
    barrier()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record(stream)
    for i in range(args.steps):
        gen.train_step_raw(pz.data_ptr(), pf.data_ptr(), pg.data_ptr(), pd.data_ptr(), pa.data_ptr(), 2000 + i)
    h1.record(stream)
    gen.sync()
    barrier()
    ms_e2e = max_over_ranks(h0.elapsed_time(h1)) / args.steps
    e2e_value = world * audio_s / (ms_e2e / 1000.0)
    h2d = (z.nbytes + f0.nbytes + g.nbytes + dldy.nbytes)
    d2h = pa.numel() * 4

    # ---- dominant kernel vs roofline (bf16 tensor peak, kernel timed alone) ----
    pk, pk_sus, hbm, pk_src = peaks()
    kms, kflops = gen.kernel_bench(0, 1, iters=20)
    achieved = kflops / (kms / 1000.0) / 1e12
    step_flops = model.train_flops_per_item(cfg, F) * B
    step_tflops = step_flops / (ms / 1000.0) / 1e12
    launches = gen.graph_kernels() * args.steps

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res, why = time_reference(args.config, F, steps=2, warmup=1)
        cpu = ({k: res[k] for k in ("value", "unit", "cores", "kind", "sample")} if res
               else {"value": None, "unavailable": why})

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16+fp16" if args.dtype == "bf16" else "fp32 (bf16x3 backward, fp16x3 forward)",
            "data": "synthetic",
            "config": {"workload": f"{args.config} NSF-HiFiGAN generator train step (fwd + bwd + AdamW), "
                                   f"batch {B}/GPU, {F} frames = {T} samples per item",
                       "global_batch": B * world, "frames": F, "samples_per_item": T,
                       "parallelism": f"dp{world}",
                       "dtype": "forward GEMMs on fp16 operand pairs (fp32-accurate), backward GEMMs on "
                                + ("bf16" if args.dtype == "bf16" else "bf16 hi + lo pairs (3 products, fp32 precision)")
                                + ", fp32 accumulation and fp32 residual streams",
                       "gemm": "tcgen05 kind::f16, fp32 accumulate; forward fp16 hi + lo/2048 pairs (3 products), "
                               "backward " + ("bf16" if args.dtype == "bf16" else
                                              "bf16 pairs: input gradients 2 MMAs (3 products), weight "
                                              "gradients 3 launches"),
                       "l2": "working set of several GB per step is larger than L2; no flush",
                       "adamw_lr": LR, "params": "reset to their init before each timed phase"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": ms_e2e},
            "gpu_launches": launches,
            "roofline": {"bound": "tensor",
                         "kernel": "tc_conv2_kernel (persistent conv) forward conv1, k=11 dil=1, stage 1 "
                                   "(51200 rows x 128 ch), split operands = 2 MMAs (3 products) per K16 step",
                         "achieved": achieved, "peak": pk, "unit": "TFLOP/s", "frac": achieved / pk,
                         "peak_source": pk_src, "traffic": TRAFFIC_BYTES, "launch_ms": kms,
                         "algorithmic_flops_per_launch": kflops,
                         "issued_tensor_tflops": achieved * 3.0,
                         "note": "achieved counts algorithmic FLOPs; the split forward issues 3x that tensor work"},
            "step_roofline": {"algorithmic_tflops": step_tflops, "peak_sustained": pk_sus,
                              "frac": step_tflops / pk_sus, "flops_per_step": step_flops},
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line))
    gen.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
