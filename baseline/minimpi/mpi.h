/* mpi.h - the subset of the MPI C interface that the reference benchmark
 * programs call, implemented by minimpi.cpp for one node.
 *
 * The reference's programs (the .cu files of src/loop and src/attention) include
 * <mpi.h> and need an MPI library to build and run; none is installed on the
 * machines this framework targets.  This header and its library let those
 * programs build UNMODIFIED with their own Makefile (MPI_HOME pointing here)
 * and run as the reference arm of the benchmark.  Names, types and signatures
 * follow the MPI standard because the programs are written against it; the
 * implementation is this library's own.
 *
 * Scope: MPI_COMM_WORLD (and MPI_Comm_split_type(SHARED), which returns the
 * world: every rank is on one node); blocking and non-blocking point-to-point
 * with in-order matching per (source, destination) pair; barrier, broadcast,
 * reduce / allreduce (MAX, MIN, SUM on int, float, double); MPI_Wtime;
 * MPI_Abort.  Buffers in device memory are moved GPU to GPU through CUDA IPC
 * (what a CUDA-aware MPI does inside a node); host buffers through POSIX
 * shared memory.
 */
#ifndef MINIMPI_MPI_H
#define MINIMPI_MPI_H

#ifdef __cplusplus
extern "C" {
#endif

typedef int MPI_Comm;
typedef int MPI_Datatype;
typedef int MPI_Op;
typedef int MPI_Info;
typedef struct minimpi_request* MPI_Request;

typedef struct MPI_Status {
  int MPI_SOURCE;
  int MPI_TAG;
  int MPI_ERROR;
  int minimpi_count_bytes;
} MPI_Status;

#define MPI_SUCCESS 0
#define MPI_ERR_OTHER 15
#define MPI_ERR_TRUNCATE 14

#define MPI_COMM_NULL ((MPI_Comm)0)
#define MPI_COMM_WORLD ((MPI_Comm)1)
#define MPI_COMM_SELF ((MPI_Comm)2)
#define MPI_COMM_TYPE_SHARED 1
#define MPI_INFO_NULL ((MPI_Info)0)
#define MPI_UNDEFINED (-32766)

#define MPI_CHAR ((MPI_Datatype)1)
#define MPI_BYTE ((MPI_Datatype)2)
#define MPI_INT ((MPI_Datatype)3)
#define MPI_FLOAT ((MPI_Datatype)4)
#define MPI_DOUBLE ((MPI_Datatype)5)
#define MPI_LONG_LONG ((MPI_Datatype)6)
#define MPI_UNSIGNED_LONG_LONG ((MPI_Datatype)7)
#define MPI_UNSIGNED ((MPI_Datatype)8)

#define MPI_MAX ((MPI_Op)1)
#define MPI_MIN ((MPI_Op)2)
#define MPI_SUM ((MPI_Op)3)

#define MPI_ANY_SOURCE (-1)
#define MPI_ANY_TAG (-1)
#define MPI_PROC_NULL (-2)
#define MPI_REQUEST_NULL ((MPI_Request)0)
#define MPI_STATUS_IGNORE ((MPI_Status*)0)
#define MPI_STATUSES_IGNORE ((MPI_Status*)0)
#define MPI_IN_PLACE ((void*)1)
#define MPI_MAX_PROCESSOR_NAME 256

#define MPI_THREAD_SINGLE 0
#define MPI_THREAD_FUNNELED 1
#define MPI_THREAD_SERIALIZED 2
#define MPI_THREAD_MULTIPLE 3

int MPI_Init(int* argc, char*** argv);
int MPI_Init_thread(int* argc, char*** argv, int required, int* provided);
int MPI_Initialized(int* flag);
int MPI_Finalize(void);
int MPI_Finalized(int* flag);
int MPI_Abort(MPI_Comm comm, int errorcode);

int MPI_Comm_rank(MPI_Comm comm, int* rank);
int MPI_Comm_size(MPI_Comm comm, int* size);
int MPI_Comm_split_type(MPI_Comm comm, int split_type, int key, MPI_Info info,
                        MPI_Comm* newcomm);
int MPI_Comm_free(MPI_Comm* comm);
int MPI_Get_processor_name(char* name, int* resultlen);

int MPI_Barrier(MPI_Comm comm);
int MPI_Bcast(void* buffer, int count, MPI_Datatype datatype, int root, MPI_Comm comm);
int MPI_Reduce(const void* sendbuf, void* recvbuf, int count, MPI_Datatype datatype, MPI_Op op,
               int root, MPI_Comm comm);
int MPI_Allreduce(const void* sendbuf, void* recvbuf, int count, MPI_Datatype datatype,
                  MPI_Op op, MPI_Comm comm);

int MPI_Send(const void* buf, int count, MPI_Datatype datatype, int dest, int tag, MPI_Comm comm);
int MPI_Recv(void* buf, int count, MPI_Datatype datatype, int source, int tag, MPI_Comm comm,
             MPI_Status* status);
int MPI_Sendrecv(const void* sendbuf, int sendcount, MPI_Datatype sendtype, int dest, int sendtag,
                 void* recvbuf, int recvcount, MPI_Datatype recvtype, int source, int recvtag,
                 MPI_Comm comm, MPI_Status* status);
int MPI_Isend(const void* buf, int count, MPI_Datatype datatype, int dest, int tag, MPI_Comm comm,
              MPI_Request* request);
int MPI_Irecv(void* buf, int count, MPI_Datatype datatype, int source, int tag, MPI_Comm comm,
              MPI_Request* request);
int MPI_Wait(MPI_Request* request, MPI_Status* status);
int MPI_Waitall(int count, MPI_Request requests[], MPI_Status statuses[]);
int MPI_Test(MPI_Request* request, int* flag, MPI_Status* status);
int MPI_Testall(int count, MPI_Request requests[], int* flag, MPI_Status statuses[]);
int MPI_Get_count(const MPI_Status* status, MPI_Datatype datatype, int* count);

double MPI_Wtime(void);

#ifdef __cplusplus
}
#endif

#endif /* MINIMPI_MPI_H */
