"""``nuvla_forge.profiling``: StepTimer, make_profiler, bandwidth_gb_s, roofline_note."""

from nuvla_forge_b200.profiling import *  # noqa: F401,F403
from nuvla_forge_b200.profiling import StepTimer, bandwidth_gb_s, make_profiler, roofline_note  # noqa: F401
