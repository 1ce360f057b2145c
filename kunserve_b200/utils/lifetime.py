"""Request lifecycle events and their JSON codec.

Parity: ``kunserve/lifetime.py:40-79``.  Unlike the reference, whose events
are defined but never emitted, the instance engine here records them when
``KUNSERVE_TRACE_LIFETIME=1`` (arrival, schedule, first token, preempt,
migrate, finish) so a run can be replayed as a timeline.
"""
import enum
import json
import time
from dataclasses import asdict, dataclass
from typing import List


class LifetimeEventType(enum.Enum):
    ISSUED = "issued"
    SCHEDULED = "scheduled"
    FIRST_TOKEN = "first_token"
    PREEMPTED = "preempted"
    MIGRATED = "migrated"
    RESHARDED = "resharded"
    FINISHED = "finished"


@dataclass
class LifetimeEvent:
    timestamp: float
    event_type: LifetimeEventType
    request_id: int = -1

    def to_json(self) -> dict:
        d = asdict(self)
        d["event_type"] = self.event_type.value
        return d

    @staticmethod
    def from_json(d: dict) -> "LifetimeEvent":
        return LifetimeEvent(d["timestamp"], LifetimeEventType(d["event_type"]),
                             d.get("request_id", -1))


def now_event(kind: LifetimeEventType, request_id: int = -1) -> LifetimeEvent:
    return LifetimeEvent(time.time(), kind, request_id)


def json_encode_lifetime_events(events: List[LifetimeEvent]) -> str:
    return json.dumps([e.to_json() for e in events])


def json_decode_lifetime_events(text: str) -> List[LifetimeEvent]:
    return [LifetimeEvent.from_json(d) for d in json.loads(text)]
