"""The autotuner's device farm, driven on the host with fake devices (no GPU):
jobs are spread over every device, a slow device takes fewer, a device that is
lost mid-sweep hands its job back and the others finish everything, a device
that fails its set-up takes no job, and when every device is lost the farm
reports the jobs left undone. The queue is the one ridge_autotune runs on
(reference loop: tools/ridge-autotune.py:94-112, which had no farm)."""

import ctypes as C

import pytest

from ridge_b200 import lib
from ridge_b200._native import RIDGE_EDEVICE, RIDGE_OK


def farm(num_jobs, num_devices, lost=-1, lost_after=0, slow=-1):
    jd = (C.c_int32 * max(num_jobs, 1))()
    per = (C.c_int32 * num_devices)()
    st = lib.ridge_farm_selftest(num_jobs, num_devices, lost, lost_after, slow, jd, per)
    return st, list(jd)[:num_jobs], list(per)


def test_every_job_done_once_across_devices():
    st, jd, per = farm(40, 4)
    assert st == RIDGE_OK
    assert all(0 <= d < 4 for d in jd)
    assert sum(per) == 40 and all(p > 0 for p in per)
    assert [jd.count(d) for d in range(4)] == per


def test_slow_device_takes_fewer_jobs():
    st, jd, per = farm(60, 3, slow=2)
    assert st == RIDGE_OK
    assert per[2] < per[0] and per[2] < per[1]


def test_lost_device_hands_its_job_back():
    st, jd, per = farm(30, 3, lost=1, lost_after=3)
    assert st == RIDGE_OK, "the surviving devices must finish every job"
    assert per[1] == 3
    assert sum(per) == 30 and all(d >= 0 for d in jd)


def test_device_failing_setup_takes_no_job():
    st, jd, per = farm(12, 2, lost=0, lost_after=-1)
    assert st == RIDGE_OK
    assert per == [0, 12] and set(jd) == {1}


@pytest.mark.parametrize("lost_after", [0, 2])
def test_all_devices_lost_reports_undone_jobs(lost_after):
    # one device only, lost after `lost_after` jobs: the rest stay undone
    st, jd, per = farm(10, 1, lost=0, lost_after=lost_after)
    assert st == RIDGE_EDEVICE
    assert per == [lost_after]
    assert sum(d == 0 for d in jd) == lost_after and jd.count(-1) == 10 - lost_after
