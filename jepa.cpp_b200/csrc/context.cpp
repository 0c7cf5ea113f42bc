// jepa_context teardown: the planners' device state, the NCCL communicator, then the stream.
#include "model.h"
#include "hplan.h"
#include "shard.h"
#include "ac.h"
#include "encoder.h"

jepa_context::~jepa_context() {
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    hplan.reset();
    ac.reset();
    enc.reset();
    shard.reset();
    if (stream) cudaStreamDestroy(stream);
}
