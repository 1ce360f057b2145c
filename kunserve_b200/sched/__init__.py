from .scheduler import ColocatedScheduler
from .admission import AdmissionMixin
