"""Run the REFERENCE's renderer glue on top of a rasterizer (test helper).

TEST INFRASTRUCTURE ONLY.  Executed as a child process by
tests/test_gpu_dropin.py:

    python tests/dropin_harness.py {ours|reference} OUT.pt

It imports the reference's own gaussian_renderer package and the utils
modules it needs (installed from the reference sources into
oracle/_ref/refsrc by oracle/build_ref.py) and runs one training step of a
two-camera batch exactly as the reference trainer drives it at world size 1
(train_internal.py: start_strategy_final ->
distributed_preprocess3dgs_and_all2all_final -> render_final ->
batched_loss_computation -> backward), on a 1-rank NCCL group.  The
rasterizer import name ``diff_gaussian_rasterization_f`` resolves to this
repository's compat package (``ours``) or to the reference build
(``reference``).  Modules the glue imports but this path does not use are
stubbed: scene.gaussian_model and scene.cameras (type names only), and
pytorch3d.transforms (imported, unused).  The model is a stand-in for
GaussianModel exposing the getters the glue reads (scene/gaussian_model.py:
248-276: exp, normalize, sigmoid, cat of the raw parameters).

Saved: the loss, per-camera images, radii and out_observe, and the gradients
of the six raw parameter tensors.
"""
import datetime
import os
import sys
import types
from argparse import Namespace

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")


def _stub_modules():
    p3d = types.ModuleType("pytorch3d")
    tr = types.ModuleType("pytorch3d.transforms")

    def quaternion_to_matrix(q):  # imported by the glue, never called on this path
        raise NotImplementedError

    tr.quaternion_to_matrix = quaternion_to_matrix
    p3d.transforms = tr
    scene = types.ModuleType("scene")
    gm = types.ModuleType("scene.gaussian_model")
    cams = types.ModuleType("scene.cameras")

    class GaussianModel:  # type name only
        pass

    class Camera:  # type name only
        pass

    gm.GaussianModel = GaussianModel
    cams.Camera = Camera
    scene.gaussian_model = gm
    scene.cameras = cams
    sys.modules.update({"pytorch3d": p3d, "pytorch3d.transforms": tr, "scene": scene,
                        "scene.gaussian_model": gm, "scene.cameras": cams})


class _Timers:
    def start(self, *_):
        pass

    def stop(self, *_):
        pass


class _Model:
    """The getters of GaussianModel the glue reads, over raw parameters."""

    def __init__(self, params):
        import torch
        self.params = params
        self._torch = torch
        self.active_sh_degree = 3

    @property
    def get_xyz(self):
        return self.params[0]

    @property
    def get_scaling(self):
        return self._torch.exp(self.params[1])

    @property
    def get_rotation(self):
        return self._torch.nn.functional.normalize(self.params[2])

    @property
    def get_opacity(self):
        return self._torch.sigmoid(self.params[3])

    @property
    def get_features(self):
        return self._torch.cat((self.params[4], self.params[5]), dim=1)


def main(which, out_path):
    sys.path.insert(0, ROOT)
    if which == "ours":
        sys.path.insert(0, os.path.join(ROOT, "blitzgs_b200", "compat"))
    else:
        sys.path.insert(0, REF)
    sys.path.insert(0, os.path.join(REF, "refsrc"))
    _stub_modules()
    import torch
    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29541")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        import diff_gaussian_rasterization_f as rast_pkg
        import utils.general_utils as U
        from gaussian_renderer import distributed_preprocess3dgs_and_all2all_final, render_final
        from gaussian_renderer.loss_distribution import batched_loss_computation
        from gaussian_renderer.workload_division import DivisionStrategyHistoryFinal, start_strategy_final
        from blitzgs_b200 import scene as S

        expect = os.path.join(ROOT, "blitzgs_b200", "compat") if which == "ours" else REF
        assert os.path.dirname(os.path.dirname(os.path.abspath(rast_pkg.__file__))) == os.path.abspath(expect), \
            rast_pkg.__file__

        sc = S.tiny(seed=0)
        sc.cameras.append(S.look_at_camera([2.2, -0.8, -2.0], [0, 0, 0], [0, -1, 0], 256, 256, 1.0, uid=1))
        H, W = 256, 256
        n = len(sc.cameras)
        U.set_args(Namespace(bsz=n, local_sampling=False, border_divpos_coeff=1.0, log_folder="/tmp",
                             log_interval=1_000_000, densify_until_iter=1_000_000_000, lambda_dssim=0.2,
                             lr_scale_loss=1.0, gaussians_distribution=True, image_distribution=True,
                             heuristic_decay=0.0, adjust_strategy_warmp_iterations=-1, no_heuristics_update=False,
                             stop_adjust_if_workloads_well_balanced=False, distributed_dataset_storage=False,
                             enable_timer=False, check_gpu_memory=False))
        U.set_cur_iter(1)
        U.set_timers(_Timers())
        U.GLOBAL_RANK, U.LOCAL_RANK, U.WORLD_SIZE = 0, 0, 1
        U.DEFAULT_GROUP = dist.group.WORLD
        U.set_block_size(16, 16, 256)
        U.set_img_size(H, W)

        params = [t.to(dev).requires_grad_(True) for t in (sc.xyz, sc.scaling, sc.rotation, sc.opacity,
                                                           sc.features_dc, sc.features_rest)]
        pc = _Model(params)
        cams = []
        for k, c in enumerate(sc.cameras):
            cc = c.to(dev)
            cams.append(Namespace(uid=k, FoVx=c.FoVx, FoVy=c.FoVy, image_height=H, image_width=W,
                                  world_view_transform=cc.world_view_transform,
                                  full_proj_transform=cc.full_proj_transform, camera_center=cc.camera_center,
                                  original_image=S.target_image(k, H, W).to(dev), image_name=f"cam{k}"))
        history = DivisionStrategyHistoryFinal(Namespace(cameras=cams), 1, 0)
        strategies, _ = start_strategy_final(cams, history)
        bg = torch.zeros(3, device=dev)
        pkg = distributed_preprocess3dgs_and_all2all_final(
            cams, pc, Namespace(debug=False), bg, batched_voxel_mask=[None] * n, batched_nearest_cameras=[None] * n,
            batched_nearest_voxel_mask=[None] * n, batched_strategies=strategies, mode="train", iterations=1)
        images, _, _, observe, _, dicts, _ = render_final(cams, pkg, strategies)
        stats = [d.get("stats_collector", {}) if isinstance(d, dict) else {} for d in pkg["batched_cuda_args"]]
        loss, _ = batched_loss_computation(images, dicts, cams, strategies, stats, 1, Namespace(scale_loss_from_iter=0))
        loss.backward()
        torch.cuda.synchronize()
        torch.save({"loss": float(loss.item()), "images": [im.detach().cpu() for im in images],
                    "radii": [d["radii"].cpu() for d in dicts], "out_observe": [o.cpu() for o in observe],
                    "grads": [p.grad.detach().cpu() for p in params],
                    "render_time_keys": [sorted(s.keys()) for s in stats]}, out_path)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2])
