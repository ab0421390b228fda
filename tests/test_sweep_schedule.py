"""CPU checks of the colour-sweep schedule (model.hpp scheduleSweep).

The step kernel sweeps one colour at a time with one lane per body, so a warp
runs as long as the body with the most hinges.  scheduleSweep hands spare
lanes of a colour to its busiest bodies.  These tests compile the host-side
model code with g++ and check the schedule's invariants: every hinge of a
colour body is stamped exactly once, helpers only split bodies whose hinge
count sets the colour's pace, and models with changing colours (body pairs)
or wide teams are left unscheduled.
"""

import json
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

PROGRAM = r"""
#include "model.hpp"
#include <cstdio>
using namespace duckb200;
int main(int argc, char **argv) {
  auto parsed = parseDuck(argv[1], 128);
  auto hm = convertModel<float>(parsed, 0.005, 10, false, 128);
  const DevModel<float> &d = hm.dev;
  printf("{\"np\": %d, \"colorStart\": [%d, %d, %d], \"colorBody\": [", d.np, d.colorStart[0], d.colorStart[1],
         d.colorStart[2]);
  for (int i = 0; i < d.colorStart[2]; ++i) printf("%s%d", i ? ", " : "", d.colorBody[i]);
  printf("], \"csrOffset\": [");
  for (int i = 0; i <= d.nb; ++i) printf("%s%d", i ? ", " : "", d.csrOffset[i]);
  printf("], \"schedules\": {");
  for (int T = 4, first = 1; T <= 32; T *= 2, first = 0) {
    scheduleSweep(hm.dev, T);
    printf("%s\"%d\": {\"scheduled\": %d, \"helpers\": [%d, %d], \"lanes\": [", first ? "" : ", ", T,
           d.sweepScheduled, d.sweepHelpers[0], d.sweepHelpers[1]);
    for (int c = 0; c < 2; ++c)
      for (int l = 0; l < 32; ++l)
        printf("%s[%d, %d, %d, %d]", c || l ? ", " : "", d.sweep[c][l][0], d.sweep[c][l][1], d.sweep[c][l][2],
               d.sweep[c][l][3]);
    printf("]}");
  }
  printf("}}\n");
}
"""


@pytest.fixture(scope="module")
def schedule_tool(tmp_path_factory):
    compiler = shutil.which("g++")
    if compiler is None:
        pytest.skip("g++ is not available")
    d = tmp_path_factory.mktemp("sched")
    (d / "sched.cpp").write_text(PROGRAM)
    exe = d / "sched"
    subprocess.run([compiler, "-std=c++17", "-O1", "-I", str(ROOT / "duck_gym_b200" / "csrc"), str(d / "sched.cpp"),
                    "-o", str(exe)], check=True)
    return exe


def run(tool, model):
    return json.loads(subprocess.run([str(tool), str(model)], check=True, capture_output=True, text=True).stdout)


def lanes_of(info, T, colour):
    return info["schedules"][str(T)]["lanes"][32 * colour:32 * colour + 32]


def test_biped_schedule_splits_the_base(schedule_tool, tmp_path):
    from duck_gym_b200 import biped

    info = run(schedule_tool, biped.write(tmp_path, seed=0))
    s8 = info["schedules"]["8"]
    assert s8["scheduled"] == 1 and s8["helpers"] == [1, 0]
    lanes = lanes_of(info, 8, 0)
    # The base (body 1, three hinges) keeps two and its helper takes one; no
    # colour-0 lane is left with more than two hinges.
    owner = [l for l in lanes[:8] if l[0] == 1 and l[3] < 32]
    helper = [l for l in lanes[:8] if l[0] == 1 and l[3] >= 32]
    assert len(owner) == 1 and len(helper) == 1
    assert owner[0][2] - owner[0][1] == 2 and helper[0][2] - helper[0][1] == 1
    assert max(l[2] - l[1] for l in lanes[:8] if l[0] >= 0) == 2
    # Teams of 16 or 32 lanes use two lanes per body and are not scheduled.
    assert info["schedules"]["16"]["scheduled"] == 0
    assert info["schedules"]["32"]["scheduled"] == 0


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
@pytest.mark.parametrize("T", [4, 8])
def test_every_hinge_stamped_once(schedule_tool, tmp_path, seed, T):
    from duck_gym_b200 import biped

    info = run(schedule_tool, biped.write(tmp_path, seed=seed))
    sched = info["schedules"][str(T)]
    cs, bodies, csr = info["colorStart"], info["colorBody"], info["csrOffset"]
    if max(cs[1] - cs[0], cs[2] - cs[1]) > T:
        assert sched["scheduled"] == 0
        return
    assert sched["scheduled"] == 1
    for colour in range(2):
        lanes = lanes_of(info, T, colour)
        assert all(l[0] == -1 for l in lanes[T:])
        covered = {}
        for lane, (body, begin, end, role) in enumerate(lanes[:T]):
            if body < 0:
                continue
            if role >= 32:  # helper: its owner names it back
                assert lanes[role - 32][0] == body and lanes[role - 32][3] == lane
            elif role >= 0:
                assert lanes[role][0] == body and lanes[role][3] == 32 + lane
            for adj in range(begin, end):
                covered.setdefault(body, []).append(adj)
        expected = {b: list(range(csr[b], csr[b + 1])) for b in bodies[cs[colour]:cs[colour + 1]]}
        assert {b: sorted(v) for b, v in covered.items()} == expected
        # A helper only exists where it lowers the colour's largest hinge count.
        if not sched["helpers"][colour]:
            assert all(l[3] == -1 for l in lanes[:T] if l[0] >= 0)


def test_pair_models_are_not_scheduled(schedule_tool, tmp_path):
    from duck_gym_b200 import biped

    path = biped.write(tmp_path, seed=0, self_contacts=True)
    info = run(schedule_tool, path)
    assert info["np"] > 0
    assert all(info["schedules"][str(T)]["scheduled"] == 0 for T in (4, 8, 16, 32))
