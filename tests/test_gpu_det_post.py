"""The det session's DB mask exit (geometry.rs:286-296 on the device) and the
device box score (geometry.rs:221-269).

With det_mask_exit the session returns the u8 mask (pred > thresh, 2x2
dilated) to the host and keeps the probability map on the device.  The mask
must equal the oracle's db_mask of the same session's probability map, the
kept map must equal the map the session returns without the exit, and box
scores computed on the kept map must equal the oracle's box_score_fast."""
import numpy as np
import pytest

import oracle as orc
import qppocr_b200 as q
from qppocr_b200 import nets

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("math", ["tf32", "3xtf32"])
def test_det_mask_exit_and_box_scores(cuda_ctx, math):
    import torch
    g, w = nets.build_det()
    g = q.optimize(g, w)
    x = nets.det_input(2, 160, 224, seed=21)
    plain = cuda_ctx.create_session(g, w, role="det", math=math)
    pred = plain.run({"x": x})[0]
    plain.close()
    s = cuda_ctx.create_session(g, w, role="det", math=math, det_mask_exit=True, mask_thresh=0.3)
    mask, dev_pred = s.run({"x": x})
    assert mask.dtype == np.uint8 and mask.shape == (2, 160, 224)
    assert isinstance(dev_pred, q.DeviceOutput) and dev_pred.shape == (2, 1, 160, 224)
    tp = dev_pred.torch()
    kept = tp.cpu().numpy()
    assert np.array_equal(kept.view(np.uint32), pred.view(np.uint32))
    assert np.array_equal(mask, orc.db_mask(pred[:, 0], 0.3, dilate=True))
    # box scores on the kept map, no host copy of it
    rng = np.random.Generator(np.random.PCG64(22))
    boxes, img = [], []
    for k in range(40):
        x0, y0 = rng.uniform(-5, 200), rng.uniform(-5, 140)
        bw, bh = rng.uniform(2, 60), rng.uniform(2, 30)
        boxes.append([[x0, y0], [x0 + bw, y0 + 0.3 * k], [x0 + bw, y0 + bh], [x0, y0 + bh]])
        img.append(k % 2)
    boxes = np.array(boxes, np.float32)
    img = np.array(img, np.int32)
    got = q.op_box_score(tp[:, 0], torch.from_numpy(boxes).cuda(), torch.from_numpy(img).cuda())
    torch.cuda.synchronize()
    ref = orc.box_scores(pred[:, 0], boxes, img)
    assert np.array_equal(got.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    del tp, dev_pred
    s.close()


def test_det_mask_exit_needs_det_role(cuda_ctx):
    g, w = nets.build_block()
    g = q.optimize(g, w)
    with pytest.raises(q.GraphError, match="det role"):
        cuda_ctx.create_session(g, w, role="other", det_mask_exit=True)
