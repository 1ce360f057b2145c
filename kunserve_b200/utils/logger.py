"""Package logger.

Same role as the reference's ``kunserve/logger.py:9-49``: one root logger for
the package that prints INFO records to stdout.  Multi-line messages are
indented so that every continuation line stays attributed to its record.
"""
import logging
import sys

_ROOT = "kunserve_b200"
_FMT = "%(levelname)s %(asctime)s.%(msecs)03d %(name)s:%(lineno)d] %(message)s"
_DATEFMT = "%m-%d %H:%M:%S"


class _IndentingFormatter(logging.Formatter):
    def format(self, record: logging.LogRecord) -> str:
        text = super().format(record)
        if record.message and "\n" in text:
            head, _, _ = text.partition(record.message)
            text = text.replace("\n", "\n" + " " * len(head))
        return text


def _root() -> logging.Logger:
    root = logging.getLogger(_ROOT)
    if not root.handlers:
        handler = logging.StreamHandler(sys.stdout)
        handler.setFormatter(_IndentingFormatter(_FMT, datefmt=_DATEFMT))
        root.addHandler(handler)
        root.setLevel(logging.INFO)
        root.propagate = False
    return root


def init_logger(name: str) -> logging.Logger:
    """Return a child of the package logger (``name`` is usually ``__name__``)."""
    _root()
    if not name.startswith(_ROOT):
        name = f"{_ROOT}.{name}"
    return logging.getLogger(name)
