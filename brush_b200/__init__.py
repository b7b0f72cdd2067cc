"""brush_b200 - B200-native (sm_100a) Gaussian-splat training step with the operator
API of debsahu/brush's render / render-bwd / loss / train crates.

The compute lives in ``libbsx.so`` (C ABI, ``include/bsx.h``); this package is
the host-side mirror of the reference's operators. There is no CPU path.
"""
from ._lib import REFINE_GRAD_THRESHOLD, REFINE_REFERENCE, BsxError, lib  # noqa: F401
from .adam import AdamGroup, AdamScaled  # noqa: F401
from .camera import Camera, focal_to_fov, fov_to_focal  # noqa: F401
from .loss import ImageLossConfig, image_loss_backward, image_loss_forward, image_loss_fused  # noqa: F401
from .primitives import get_tile_offsets, prefix_sum, radix_argsort  # noqa: F401
from .render import RasterPass, RenderOutput, SplatRenderMode, render, render_splats  # noqa: F401
from .render_bwd import SplatGrads, project_bwd, project_bwd_ref, rasterize_bwd, rasterize_bwd_ref  # noqa: F401
from .splats import Splats  # noqa: F401
from .train import RefineConfig, SplatTrainer, TrainConfig  # noqa: F401
