"""Generate tests/golden/ref_cfg0.{npz,json}: the reference's OWN CPU kernels run on a seeded
config-0 scene (2,048 Gaussians, SH deg 0, 256x256 pinhole), so machines without the reference
tree can still pin the oracle and the GPU path to the reference's outputs.

Needs oracle/_ref/libsplatx_ref.so (``make -C oracle ref`` where the reference tree exists):

    python tests/golden/make_ref_vectors.py
"""
from __future__ import annotations

import json
import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "splatx-metal_b200"))

import oracle  # noqa: E402
from splatx_cuda.scene import small_scene  # noqa: E402


def main():
    rb = oracle.RefBackend()
    scene, cam = small_scene(seed=11, n=2048, sh_degree=0)
    s = np.exp(scene.scales).astype(np.float32)
    o = (np.float32(1) / (np.float32(1) + np.exp(-scene.opacities).astype(np.float32))).astype(np.float32)
    tw = th = 16
    p = rb.projection_fused_fwd(scene.means, cam.viewmat, cam.K, cam.width, cam.height,
                                quats=scene.quats, scales=s, opacities=o)
    it = rb.isect_tiles(p.means2d, p.radii, p.depths, 1, scene.count, 16, tw, th, conics=p.conics,
                        opacities=o)
    st = rb.sort_isect(it.isect_ids, it.flatten_ids, 32 + it.tile_n_bits + it.image_n_bits)
    off = rb.isect_offset_encode(st.keys_sorted, it.n_isects, 1, tw, th)
    colors = np.random.default_rng(12).uniform(0, 1, scene.count * 3).astype(np.float32)
    ras = rb.rasterize_fwd(p.means2d, p.conics, colors, o, off, st.values_sorted, 1, scene.count,
                           it.n_isects, cam.width, cam.height, 16, tw, th)
    out = pathlib.Path(__file__).resolve().parent
    np.savez_compressed(out / "ref_cfg0.npz", means=scene.means, quats=scene.quats, scales=s,
                        opacities=o, viewmat=cam.viewmat, K=cam.K, colors=colors, radii=p.radii,
                        means2d=p.means2d, depths=p.depths, conics=p.conics,
                        tiles_per_gauss=it.tiles_per_gauss, isect_ids=it.isect_ids,
                        flatten_ids=it.flatten_ids, isect_ids_sorted=st.keys_sorted,
                        flatten_ids_sorted=st.values_sorted, offsets=off,
                        render_colors=ras.render_colors, render_alphas=ras.render_alphas,
                        last_ids=ras.last_ids)
    meta = {"source": "splatx-metal CpuKernels.cpp (projection_fused_fwd_cpu, isect_tiles_cpu "
                      "AccuTile, sort_isect_cpu, isect_offset_encode_cpu, rasterize_fwd_cpu) built "
                      "by oracle/Makefile from the reference tree",
            "N": scene.count, "width": cam.width, "height": cam.height, "tile_width": tw,
            "tile_height": th, "n_isects": int(it.n_isects), "scene_seed": 11, "colors_seed": 12}
    (out / "ref_cfg0.json").write_text(json.dumps(meta, indent=1) + "\n")
    print(meta)


if __name__ == "__main__":
    main()
