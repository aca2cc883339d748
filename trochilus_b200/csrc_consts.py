"""The exponential's exception table as Python data, read from csrc/expf_consts.h."""
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))


def exceptions():
    text = open(os.path.join(HERE, "csrc", "expf_consts.h")).read()
    return [(int(a, 16), int(b, 16)) for a, b in re.findall(r"\{0x([0-9a-f]+)u, 0x([0-9a-f]+)u\}", text)]
