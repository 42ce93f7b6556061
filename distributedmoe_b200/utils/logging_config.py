"""Named loggers for the package (the reference's ``utils/logging_config.py:172-180`` API).

Unlike the reference module, importing this does not configure handlers or create log
files; the application configures logging.  ``LOG_LEVEL`` sets the package level."""

from __future__ import annotations

import logging
import os
from logging import LoggerAdapter
from typing import Dict, Optional, Union

_root = logging.getLogger("dist_moe")
if os.getenv("LOG_LEVEL"):
    _root.setLevel(os.getenv("LOG_LEVEL", "WARNING").upper())


def get_logger(name: str, context: Optional[Dict[str, str]] = None) -> Union[logging.Logger, LoggerAdapter]:
    logger = logging.getLogger(name)
    return LoggerAdapter(logger, context) if context else logger
