"""Extract the golden vectors of ThreeDGaussianSplatting.jl's own test suite into
reference_golden.json (committed beside this script).

The reference is Julia and cannot run in this image, so its tests are read as text: every
number below comes from the literal arrays in the reference's test files, located by the
statements that hold them. Run from the repository root with the reference checkout at
$GS3D_REFERENCE_ROOT (default: the directory `reference` beside the repository):

    python tests/golden/extract_golden.py
"""
from __future__ import annotations

import json
import os
import re
from pathlib import Path

ROOT = Path(os.environ.get("GS3D_REFERENCE_ROOT",
                           Path(__file__).resolve().parents[3] / "reference"))
OUT = Path(__file__).resolve().parent / "reference_golden.json"
NUM = re.compile(r"[-+]?(?:\d+\.\d*|\.\d+|\d+)(?:[eE][-+]?\d+)?")


def strip_comments(text: str) -> str:
    return "\n".join(line.split("#", 1)[0] for line in text.splitlines())


def bracket_block(text: str, start: int) -> tuple[str, int]:
    """Text of the bracket group opening at text[start] ('[' or '(')."""
    open_ch = text[start]
    close_ch = {"[": "]", "(": ")"}[open_ch]
    depth = 0
    for i in range(start, len(text)):
        if text[i] == open_ch:
            depth += 1
        elif text[i] == close_ch:
            depth -= 1
            if depth == 0:
                return text[start + 1:i], i + 1
    raise ValueError("unbalanced brackets")


def top_level_split(text: str) -> list[str]:
    parts, depth, cur = [], 0, []
    for ch in text:
        if ch in "[(":
            depth += 1
        elif ch in "])":
            depth -= 1
        if ch == "," and depth == 0:
            parts.append("".join(cur))
            cur = []
        else:
            cur.append(ch)
    if "".join(cur).strip():
        parts.append("".join(cur))
    return parts


def numbers(text: str) -> list[float]:
    return [float(x) for x in NUM.findall(text)]


def array_after(text: str, marker: str, occurrence: int = 0) -> list[float]:
    """Numbers of the first Int32[...] / Float32[...] / Bool[...] / [...] literal after marker."""
    pos = -1
    for _ in range(occurrence + 1):
        pos = text.index(marker, pos + 1)
    m = re.compile(r"(?:Int32|Float32|Bool)?\[").search(text, pos + len(marker))
    body, _ = bracket_block(text, m.end() - 1)
    return numbers(body)


def forward_core(src: str) -> dict:
    t = strip_comments(src)
    out = {
        "keep_gaussians": array_after(t, "keep_gaussians = CuVector(Bool"),
        "fgidx_to_gidx": array_after(t, "@test fgidx_to_gidx[1:nb_fgaussians] =="),
        "nb_overlapped_tiles": array_after(t, "buffers.f2dgs_nb_overlapped_tiles .= CuVector("),
        "intersected_tile_ranges": array_after(t, "buffers.f2dgv.intersected_tile_ranges .= CuArray(reshape("),
        "dfgidx_to_fgidx": array_after(t, "@test buffers.dfgidx_to_fgidx =="),
        "sdfgidx_to_fgidx": array_after(t, "@test buffers.sdfgidx_to_fgidx =="),
        "tiles_end_sdfgidx": array_after(t, "@test buffers.tiles_end_sdfgidx =="),
        "depths": [1, 2, 3, 4, 5],
        "tiling": {"screen": [2, 2], "tile": [1, 1]},
    }
    rgb = {}
    for m in re.finditer(r"rgb_image_(\d)\[:,\s*(\d+),\s*(\d+)\],\s*\[([^\]]+)\]", t):
        deg, v, u, vals = m.group(1), int(m.group(2)), int(m.group(3)), numbers(m.group(4))
        rgb.setdefault(deg, []).append({"v": v, "u": u, "rgb": vals})
    out["rgb_pixels"] = rgb
    return out


def backward_core(src: str) -> dict:
    t = strip_comments(src)
    start = t.index("ref_gradients = Dict(")
    body, _ = bracket_block(t, start + len("ref_gradients = Dict"))
    result = {}
    for m in re.finditer(r"(\d)\s*=>\s*Dict\(", body):
        deg = m.group(1)
        inner, _ = bracket_block(body, m.end() - 1)
        entries = {}
        for km in re.finditer(r'"(\w+)"\s*=>\s*\[', inner):
            arr, _ = bracket_block(inner, km.end() - 1)
            entries[km.group(1)] = [numbers(e) for e in top_level_split(arr)]
        result[deg] = entries
    return {"gradients": result, "gt_gray": 0.5}


def training(src: str) -> dict:
    t = strip_comments(src)
    return {
        "should_prune": array_after(t, "should_prune_cpu   = Bool"),
        "should_densify": array_after(t, "should_densify_cpu = Bool"),
        "new_gaussian_counts": array_after(t, "@test new_gaussian_counts_cpu =="),
        "new_gaussian_counts_cs": array_after(t, "@test new_gaussian_counts_cs_cpu =="),
        "ngidx_to_gidx": array_after(t, "@test ngidx_to_gidx_cpu =="),
        "should_clone": array_after(t, "should_clone = cu(Bool"),
        "should_split": array_after(t, "should_split = cu(Bool"),
        "means_after_adc_ids": array_after(t, "get_mean_sv.(view(gaussians_cpu,"),
        "means_after_adc": array_after(t, "== repeat(Float32"),
        "scaling_after_adc": array_after(t, "≈ repeat(Float32"),
        "moments_after_adc": array_after(t, "== repeat(reshape(Float32"),
        "original_fgidx_to_gidx": array_after(t, "original_fgidx_to_gidx_cpu ="),
        "adjusted_fgidx_to_gidx": array_after(t, "nb_fgaussians) == cu"),
        "splits_second_copies_ids": array_after(t, "splits_second_copies_ids ="),
        "filtered_out_indices": array_after(t, "filtered_out_indices ="),
        "adam": {"beta1": 0.5, "beta2": 0.5, "epsilon": 0.0, "lr": 1.0, "lr_sh_rest": 10.0,
                 "checked": [[8, 6, 2], [9, 8, 3]]},
        "opacity_reset_max": 0.8,
    }


def main() -> None:
    data = {
        "source": "ThreeDGaussianSplatting.jl test suite (test/forward_core.jl, "
                  "test/backward_core.jl, test/training.jl), read as text",
        "forward_core": forward_core((ROOT / "test/forward_core.jl").read_text()),
        "backward_core": backward_core((ROOT / "test/backward_core.jl").read_text()),
        "training": training((ROOT / "test/training.jl").read_text()),
    }
    OUT.write_text(json.dumps(data, indent=1) + "\n")
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
