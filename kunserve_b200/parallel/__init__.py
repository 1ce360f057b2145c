from .topology import Topology, COMMS
