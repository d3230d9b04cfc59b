from .timers import DeviceTimer, HostTimer, max_over_ranks  # noqa: F401
from .logging import log_json, get_logger  # noqa: F401
