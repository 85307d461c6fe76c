! Drop-in replacement of module llama_model_gpu (llama_model_gpu.f90) over libq35.so.
! Same public names.  init_llama_model_gpu allocates the host model as the reference does
! (embeddings, 80 layers with unit norms, RoPE tables and KV caches, final norm, LM head);
! the caller then loads weights into those arrays; the first forward_llama_gpu uploads the
! whole model to the GPU (one libq35 model of max_batch_size sequences) and runs there,
! continuing on the KV cache like the reference.  After editing host weights call
! cleanup_llama_model_gpu and initialise again, or load them before the first forward.
! Every procedure takes an optional stat=; without it a failure stops with libq35's
! message (q35_status).
! Compile after llama_model.f90.
module llama_model_gpu
    use iso_c_binding, only: c_int, c_int32_t, c_ptr, c_null_ptr, c_associated, c_loc
    use iso_fortran_env, only: int32, real32
    use q35_status, only: q35_check
    use q35_model_api, only: q35_model_forward, q35_model_destroy
    use transformer_layer
    use llama_model, only: model_device_create
    implicit none
    private
    public :: LLaMAModelGPU, init_llama_model_gpu, forward_llama_gpu, cleanup_llama_model_gpu

    ! llama_model_gpu.f90:14-16
    integer(int32), parameter :: NUM_LAYERS = 80
    integer(int32), parameter :: VOCAB_SIZE = 32000
    integer(int32), parameter :: MAX_SEQ_LEN = 2048

    ! llama_model_gpu.f90:26-34, plus the device handle and the batch it was made for
    type :: LLaMAModelGPU
        real(real32), allocatable :: token_embeddings(:,:)
        type(TransformerLayer), allocatable :: layers(:)
        real(real32), allocatable :: final_norm(:)
        real(real32), allocatable :: output_weights(:,:)
        integer(int32) :: num_layers = 0
        integer(int32) :: max_seq_len = 0
        logical :: gpu_initialized = .false.
        integer(int32) :: max_batch = 1
        type(c_ptr) :: handle = c_null_ptr
    end type LLaMAModelGPU

contains

    ! llama_model_gpu.f90:41-113
    subroutine init_llama_model_gpu(model, max_batch_size)
        type(LLaMAModelGPU), intent(inout) :: model
        integer(int32), intent(in), optional :: max_batch_size
        integer(int32) :: i
        model%max_batch = 1
        if (present(max_batch_size)) model%max_batch = max(1, max_batch_size)
        print *, "=========================================="
        print *, "Initializing GPU LLaMA 70B (libq35, B200)"
        print *, "=========================================="
        print *, "  Layers:", NUM_LAYERS
        print *, "  Hidden dim:", HIDDEN_DIM
        print *, "  Vocab size:", VOCAB_SIZE
        print *, "  Max seq len:", MAX_SEQ_LEN
        print *, "  Max batch size:", model%max_batch
        model%num_layers = NUM_LAYERS
        model%max_seq_len = MAX_SEQ_LEN
        allocate(model%token_embeddings(VOCAB_SIZE, HIDDEN_DIM))
        model%token_embeddings = 0.0
        allocate(model%layers(NUM_LAYERS))
        do i = 1, NUM_LAYERS
            allocate(model%layers(i)%attn_norm(HIDDEN_DIM))
            allocate(model%layers(i)%ffn_norm(HIDDEN_DIM))
            model%layers(i)%attn_norm = 1.0
            model%layers(i)%ffn_norm = 1.0
            call init_rope_freqs(model%layers(i), MAX_SEQ_LEN)
            call init_kv_cache(model%layers(i), MAX_SEQ_LEN)
        end do
        allocate(model%final_norm(HIDDEN_DIM))
        allocate(model%output_weights(HIDDEN_DIM, VOCAB_SIZE))
        model%final_norm = 1.0
        model%output_weights = 0.0
        model%gpu_initialized = .true.
    end subroutine init_llama_model_gpu

    ! llama_model_gpu.f90:118-158
    subroutine forward_llama_gpu(model, token_ids, output_logits, seq_len, stat)
        type(LLaMAModelGPU), intent(inout), target :: model
        integer(int32), intent(in) :: token_ids(:)
        real(real32), intent(out), target, contiguous :: output_logits(:,:)
        integer(int32), intent(in), value :: seq_len
        integer, intent(out), optional :: stat
        integer :: st
        integer(int32) :: l
        if (present(stat)) stat = 0
        if (.not. model%gpu_initialized) then
            if (present(stat)) then
                stat = 6
                return
            end if
            error stop "forward_llama_gpu: GPU model not initialized (init_llama_model_gpu)"
        end if
        if (.not. c_associated(model%handle)) then
            call model_device_create(model%layers, model%token_embeddings, model%final_norm, model%output_weights, &
                                     model%num_layers, model%max_seq_len, model%max_batch, model%handle, st)
            if (st /= 0) then
                call q35_check(int(st, c_int), "forward_llama_gpu", stat)
                return
            end if
        end if
        if (size(output_logits, 1) /= seq_len .or. size(token_ids) < seq_len) then
            if (present(stat)) then
                stat = 1
                return
            end if
            error stop "forward_llama_gpu: output_logits must be (seq_len, vocab) and token_ids hold seq_len ids"
        end if
        st = q35_model_forward(model%handle, 0_c_int32_t, token_ids, seq_len, c_loc(output_logits))
        if (st == 0) then
            do l = 1, model%num_layers
                model%layers(l)%cache_pos = model%layers(l)%cache_pos + seq_len
            end do
        end if
        call q35_check(int(st, c_int), "forward_llama_gpu", stat)
    end subroutine forward_llama_gpu

    ! llama_model_gpu.f90:163-190
    subroutine cleanup_llama_model_gpu(model)
        type(LLaMAModelGPU), intent(inout) :: model
        integer(int32) :: i
        integer(c_int) :: st
        if (c_associated(model%handle)) then
            st = q35_model_destroy(model%handle)
            model%handle = c_null_ptr
        end if
        if (allocated(model%token_embeddings)) deallocate(model%token_embeddings)
        if (allocated(model%final_norm)) deallocate(model%final_norm)
        if (allocated(model%output_weights)) deallocate(model%output_weights)
        if (allocated(model%layers)) then
            do i = 1, size(model%layers)
                call release_layer(model%layers(i))
            end do
            deallocate(model%layers)
        end if
        model%gpu_initialized = .false.
    end subroutine cleanup_llama_model_gpu

end module llama_model_gpu
