"""Host logic of bench.py that needs no GPU: both arms report one workload config."""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402


def _args(streams=64, backbone='shared'):
    return argparse.Namespace(group=8, prompt=512, streams=streams, lanes=8, backbone=backbone)


def test_frame_config_keys_and_backbone_mode():
    a = _args()
    c = bench.frame_config(a, 2, 64, 8, True, 18, [513, 540])
    assert c['streams'] == 128 and c['streams_per_gpu'] == 64 and c['parallelism'] == 'replica x2'
    assert c['backbone'] == 'shared' and 'row groups of 64' in c['workload']
    assert set(c) >= {'workload', 'streams', 'streams_per_gpu', 'step', 'streams_per_launch', 'prompt_len',
                      'kv_len', 'parallelism', 'lanes', 'backbone', 'lane_sms', 'l2', 'cb0', 'prefill'}
    c2 = bench.frame_config(a, 1, 128, 8, False, 18, [513, 540])
    assert c2['backbone'] == 'lanes' and 'a backbone graph per 8 streams' in c2['workload']


def test_reference_and_flashb_arms_share_the_workload():
    """The reference arm derives its config from the same arguments as the flashb arm (kv_len and lane_sms aside,
    which describe the run)."""
    a = _args()
    flashb = bench.frame_config(a, 1, 64, 8, True, 18, [513, 546])
    ref = bench.frame_config(a, 1, a.streams, 8, a.backbone == 'shared' and 2 * a.streams <= 128, None, [513, 515])
    for k in flashb:
        if k not in ('kv_len', 'lane_sms'):
            assert flashb[k] == ref[k], k
