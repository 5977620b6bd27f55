/*
 * ekv_vmm.h — chunked CUDA virtual-memory backing exported by libekv_b200.so.
 *
 * The entry points keep the names, argument meaning and error convention of the
 * reference's native/elastic_vmm.cpp C ABI (native/elastic_vmm.cpp:316-369), so
 * the reference's ctypes loader (elastic_kv/backing.py:19-52) can bind this
 * library through ELASTIC_VMM_LIBRARY unchanged.  The implementation is new:
 * driver entry points are resolved at run time through the CUDA runtime (the
 * library has no link-time dependency on libcuda), chunk state is a dense
 * per-chunk table sized from the reservation, and zero-fill of new chunks runs
 * on a private non-blocking stream.
 *
 * Semantics:
 *   ev_create     reserve ceil(capacity/chunk)*chunk bytes of VA on `device`
 *                 (chunk must be a multiple of the VMM granularity); NULL on error.
 *   ev_ensure     map + zero every listed chunk that is not yet mapped and wait for
 *                 the zero fill (also of earlier ev_precommit chunks); all-or-nothing:
 *                 on failure the chunks mapped by this call are released again.
 *   ev_precommit  like ev_ensure but returns before the zero fill completes; a
 *                 later ev_ensure / ev_drop waits for it.
 *   ev_drop       unmap and release every listed chunk that is mapped.  The
 *                 caller guarantees no in-flight GPU work touches them.
 *   ev_base / ev_backed / ev_reserved / ev_granularity
 *                 reservation base address, committed bytes, reserved bytes and
 *                 VMM granularity; UINT64_MAX on error.
 *   ev_poisoned   1 when a failure left the backing in an uncertain state (every
 *                 later mutating call fails), 0 otherwise, -1 on error.
 *   ev_close      synchronize the context, release everything, free the handle.
 *   ev_error      thread-local message of the last failure.
 *
 * Additions without a reference counterpart (the reference behaviour is the
 * default, a spare limit of 0):
 *   ev_set_spare  keep up to `chunks` physical handles that ev_drop unmaps, for
 *                 ev_ensure / ev_precommit to map again instead of creating new
 *                 ones (on B200 cuMemRelease + cuMemCreate cost ~300 us per 2 MiB
 *                 chunk); lowering the limit releases the surplus now.  Kept
 *                 handles hold device memory but are not counted by ev_backed.
 *   ev_spare      bytes held by kept handles; UINT64_MAX on error.
 */
#ifndef EKV_VMM_H
#define EKV_VMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* native/elastic_vmm.cpp:318 */
void* ev_create(int device, uint64_t capacity_bytes, uint64_t chunk_bytes);
/* native/elastic_vmm.cpp:326 */
int ev_ensure(void* handle, const uint64_t* indices, size_t count);
/* native/elastic_vmm.cpp:333 */
int ev_precommit(void* handle, const uint64_t* indices, size_t count);
/* native/elastic_vmm.cpp:340 */
int ev_drop(void* handle, const uint64_t* indices, size_t count);
/* native/elastic_vmm.cpp:347-352 */
uint64_t ev_base(void* handle);
uint64_t ev_backed(void* handle);
uint64_t ev_reserved(void* handle);
uint64_t ev_granularity(void* handle);
/* native/elastic_vmm.cpp:353 */
int ev_poisoned(void* handle);
/* native/elastic_vmm.cpp:357 */
const char* ev_error(void);
/* native/elastic_vmm.cpp:359 */
int ev_close(void* handle);
/* no reference counterpart (see above) */
int ev_set_spare(void* handle, uint64_t chunks);
uint64_t ev_spare(void* handle);

#ifdef __cplusplus
}
#endif

#endif /* EKV_VMM_H */
