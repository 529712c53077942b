"""Environment preflight: ``python -m h3_a100.preflight [--config X] [--json out.json]``.

Counterpart of the reference's ``scripts/preflight.py`` (``:53-179``), which
checks LightX2V/Diffusers pins, the FA3 binding, GPUs, model layout and host
RAM.  Here the stack is self-contained, so the checks are: Python / torch /
CUDA versions, B200 count and compute capability 10.0, the compiled sm_100a
extension, NCCL availability, peer access (P2P over NVLink) between every GPU
pair, symmetric-memory support, host RAM against what boundary staging will
pin, and (with ``--config``) the config's derived sizes.  Emits one JSON
report and exits non-zero on a hard failure.
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import sys

import torch


def _host_ram_gib() -> float:
    try:
        import psutil

        return psutil.virtual_memory().total / 1024**3
    except Exception:  # noqa: BLE001 - psutil is optional
        with open("/proc/meminfo") as fh:
            for line in fh:
                if line.startswith("MemTotal:"):
                    return int(line.split()[1]) / 1024**2
    return 0.0


def run(config_path: str | None = None) -> dict:
    report: dict = {"ok": True, "errors": [], "warnings": [], "checks": {}}
    c = report["checks"]
    c["python"] = platform.python_version()
    c["torch"] = torch.__version__
    c["cuda_runtime"] = torch.version.cuda
    c["cuda_available"] = torch.cuda.is_available()
    try:
        from . import _C  # noqa: F401

        c["extension"] = "h3_a100._C loaded"
    except ImportError as exc:
        c["extension"] = f"missing: {exc}"
        report["errors"].append("sm_100a extension not built (python setup.py build_ext --inplace)")
    c["nccl"] = torch.distributed.is_nccl_available()
    if torch.cuda.is_available():
        n = torch.cuda.device_count()
        gpus = [{"index": i, "name": torch.cuda.get_device_name(i),
                 "capability": list(torch.cuda.get_device_capability(i)),
                 "memory_gib": round(torch.cuda.get_device_properties(i).total_memory / 1024**3, 1)}
                for i in range(n)]
        c["gpus"] = gpus
        bad = [g for g in gpus if tuple(g["capability"]) != (10, 0)]
        if bad:
            report["errors"].append(f"GPUs without compute capability 10.0 (sm_100a): {[g['name'] for g in bad]}")
        p2p = {f"{a}->{b}": torch.cuda.can_device_access_peer(a, b) for a in range(n) for b in range(n) if a != b}
        c["peer_access"] = p2p
        if n > 1 and not all(p2p.values()):
            report["warnings"].append("not every GPU pair has peer access; distributed.comm=p2p will not work")
        try:
            import torch.distributed._symmetric_memory as symm  # noqa: F401

            c["symmetric_memory"] = True
        except ImportError:
            c["symmetric_memory"] = False
            report["warnings"].append("torch symmetric memory unavailable; use distributed.comm=nccl")
    else:
        report["warnings"].append("no CUDA device visible (CPU-only: kernels.backend must be torch)")
    ram = _host_ram_gib()
    c["host_ram_gib"] = round(ram, 1)
    if config_path:
        from .config import load_config
        from .models.shared_backbone import dit_config_from, sequence_tokens

        cfg = load_config(config_path)
        dit = dit_config_from(cfg)
        tokens = sequence_tokens(cfg)
        boundary = tokens * dit.hidden * 2
        ranks = int(os.environ.get("LOCAL_WORLD_SIZE", max(1, torch.cuda.device_count())))
        pinned = boundary * dit.num_blocks * ranks / 1024**3
        c["config"] = {"path": config_path, "tokens": tokens, "boundary_bytes": boundary,
                       "frozen_params": dit.param_counts()["frozen_total"],
                       "pinned_boundary_gib_per_node": round(pinned, 1)}
        if ram and pinned > 0.5 * ram:
            report["warnings"].append(f"host boundary slabs would need {pinned:.0f} GiB of {ram:.0f} GiB RAM: "
                                      "staging_target auto keeps them in HBM instead")
    report["ok"] = not report["errors"]
    return report


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--config", default=None)
    p.add_argument("--json", default=None, help="also write the report here")
    args = p.parse_args(argv)
    report = run(args.config)
    text = json.dumps(report, indent=1)
    print(text)
    if args.json:
        with open(args.json, "w") as fh:
            fh.write(text)
    return 0 if report["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
