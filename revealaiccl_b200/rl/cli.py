"""Train / test CLIs of the schedule-search policy (scripts/train.py:67-215, scripts/test.py).

    python -m revealaiccl_b200.rl.cli train --topologies Rear4GPU --epochs 5 --output-dir runs/
    python -m revealaiccl_b200.rl.cli test --checkpoint runs/Rear4GPU_best.pth --topologies Rear4GPU

Checkpoint layout (kept compatible in keys and file names):
``{"epoch", "model_state_dict", "optimizer_state_dict", "best_score", "config",
"topologies"}`` written to ``{output_dir}/{model_name}_best.pth``,
``{model_name}_epoch{N}.pth`` and ``{model_name}_final.pth`` where
``model_name`` is the topology name or ``multi_topology``.  Resume restores
model, optimizer, ``epoch + 1`` and the best score, and also accepts a bare
state dict.
"""

from __future__ import annotations

import argparse
import json
import os
from typing import Any

import numpy as np
import torch

from ..models.policy import SlotLevelPolicy
from ..topology.loader import ensure_bundled, load_topology_info
from .ppo import evaluate_model, get_config, train_epoch
from .scenarios import generate_train_test_split


def model_name_for(topologies: list[str]) -> str:
    return topologies[0] if len(topologies) == 1 else "multi_topology"


def save_checkpoint(path: str, *, epoch: int, model, optimizer, best_score: float, config: dict,
                    topologies: list[str]) -> None:
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    torch.save({"epoch": int(epoch), "model_state_dict": model.state_dict(),
                "optimizer_state_dict": optimizer.state_dict(), "best_score": float(best_score),
                "config": dict(config), "topologies": list(topologies)}, path)


def load_checkpoint(path: str, model, optimizer=None, *, device="cpu") -> tuple[int, float]:
    """Returns (start_epoch, best_score); accepts a full checkpoint or a bare state dict."""
    ck = torch.load(path, map_location=device, weights_only=False)
    if isinstance(ck, dict) and "model_state_dict" in ck:
        model.load_state_dict(ck["model_state_dict"], strict=True)
        if optimizer is not None and "optimizer_state_dict" in ck:
            optimizer.load_state_dict(ck["optimizer_state_dict"])
        return int(ck.get("epoch", -1)) + 1, float(ck.get("best_score", -float("inf")))
    model.load_state_dict(ck, strict=True)
    return 0, -float("inf")


def run_train(args) -> dict[str, Any]:
    cfg = get_config()
    for k in ("epochs", "ppo_epochs", "batch_target", "hidden_dim", "mini_batch_size"):
        v = getattr(args, k, None)
        if v is not None:
            cfg[k] = v
    if args.lr is not None:
        cfg["lr"] = args.lr
    device = torch.device(args.device)
    torch.manual_seed(args.seed)
    np.random.seed(args.seed)
    ensure_bundled()
    topos = {n: load_topology_info(n) for n in args.topologies}
    train, test = generate_train_test_split(topos, num_train=args.num_train, num_test=args.num_test, seed=args.seed,
                                            cache_dir=args.cache_dir, T=args.T)
    model = SlotLevelPolicy(5, 2, 5, 2, cfg["hidden_dim"]).to(device)
    opt = torch.optim.Adam(model.parameters(), lr=cfg["lr"])
    name = model_name_for(args.topologies)
    start, best = 0, -float("inf")
    if args.resume:
        start, best = load_checkpoint(args.resume, model, opt, device=device)
    history = []
    for epoch in range(start, cfg["epochs"]):
        pl, vl, ent, rew = train_epoch(model, opt, train, device, cfg, epoch, cfg["epochs"], seed=args.seed + epoch,
                                       log=lambda *a: None)
        rec = {"epoch": epoch, "policy_loss": pl, "value_loss": vl, "entropy": ent, "reward": rew}
        if (epoch + 1) % args.eval_interval == 0 or epoch + 1 == cfg["epochs"]:
            score, steps = evaluate_model(model, test, device, log=lambda *a: None)
            rec.update(score=score, steps=steps)
            if score > best:
                best = score
                save_checkpoint(os.path.join(args.output_dir, f"{name}_best.pth"), epoch=epoch, model=model,
                                optimizer=opt, best_score=best, config=cfg, topologies=args.topologies)
        if (epoch + 1) % args.save_interval == 0:
            save_checkpoint(os.path.join(args.output_dir, f"{name}_epoch{epoch + 1}.pth"), epoch=epoch, model=model,
                            optimizer=opt, best_score=best, config=cfg, topologies=args.topologies)
        history.append(rec)
        print(json.dumps(rec), flush=True)
    save_checkpoint(os.path.join(args.output_dir, f"{name}_final.pth"), epoch=cfg["epochs"] - 1, model=model,
                    optimizer=opt, best_score=best, config=cfg, topologies=args.topologies)
    return {"best_score": best, "history": history}


def run_test(args) -> dict[str, Any]:
    device = torch.device(args.device)
    ck = torch.load(args.checkpoint, map_location=device, weights_only=False)
    cfg = ck.get("config", get_config()) if isinstance(ck, dict) else get_config()
    model = SlotLevelPolicy(5, 2, 5, 2, cfg.get("hidden_dim", 128)).to(device)
    load_checkpoint(args.checkpoint, model, device=device)
    ensure_bundled()
    topos = {n: load_topology_info(n) for n in args.topologies}
    _, test = generate_train_test_split(topos, num_train=0, num_test=args.num_test, seed=args.seed, T=args.T)
    score, steps = evaluate_model(model, test, device)
    out = {"score": score, "steps": steps, "problems": len(test)}
    print(json.dumps(out), flush=True)
    if args.xml_dir:
        from .decoder import SlotDecoder, rollout
        from .xml_export import export_problem_schedule

        os.makedirs(args.xml_dir, exist_ok=True)
        for sid, prob in test[: args.xml_limit]:
            sched, _ = rollout(SlotDecoder(prob.topology_info), model, prob, train=False)
            export_problem_schedule(prob, sched, os.path.join(args.xml_dir, sid.replace(":", "_") + ".xml"), name=sid)
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="revealaiccl_b200.rl.cli")
    sub = ap.add_subparsers(dest="cmd", required=True)
    for cmd in ("train", "test"):
        p = sub.add_parser(cmd)
        p.add_argument("--topologies", nargs="+", default=["Rear4GPU"])
        p.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
        p.add_argument("--seed", type=int, default=42)
        p.add_argument("--T", type=int, default=20)
        p.add_argument("--num-test", type=int, default=20)
    tr = sub.choices["train"]
    tr.add_argument("--epochs", type=int)
    tr.add_argument("--ppo-epochs", dest="ppo_epochs", type=int)
    tr.add_argument("--batch-target", dest="batch_target", type=int)
    tr.add_argument("--hidden-dim", dest="hidden_dim", type=int)
    tr.add_argument("--mini-batch-size", dest="mini_batch_size", type=int)
    tr.add_argument("--lr", type=float)
    tr.add_argument("--num-train", type=int, default=80)
    tr.add_argument("--output-dir", default="checkpoints")
    tr.add_argument("--cache-dir", default=None)
    tr.add_argument("--resume", default=None)
    tr.add_argument("--eval-interval", type=int, default=5)
    tr.add_argument("--save-interval", type=int, default=10)
    te = sub.choices["test"]
    te.add_argument("--checkpoint", required=True)
    te.add_argument("--xml-dir", default=None)
    te.add_argument("--xml-limit", type=int, default=5)
    args = ap.parse_args(argv)
    run_train(args) if args.cmd == "train" else run_test(args)


if __name__ == "__main__":
    main()
