from .actors import (ActorHandle, LocalActor, ThreadActor, ProcessActor, ActorDiedError, RemoteError,
                     make_actor, get, aw, ray_available)
